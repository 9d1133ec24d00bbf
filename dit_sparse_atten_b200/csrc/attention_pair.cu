// (a) Block-sparse flash attention, two query blocks per CTA (128-token
// blocks), for sm_100a.
//
// Reference semantics: FlexAttention with full blocks only, as driven by
// attention_backends/flex.py:308-355 (route -> BlockMask) and :379-399;
// equivalently the gather/softmax/PV of attention_backends/sparse.py:670-751.
// A query in block qb of head h attends to every valid key (< T) in the key
// blocks listed in its CSR row.
//
// Why two query blocks: a CTA with one 128-row query tile streams 64 KB of K
// and V from L2 per kept key block, which on B200 takes longer than the
// block's 1,024 tensor cycles.  Adjacent query blocks share most of their
// routed key blocks, so this kernel gives a CTA query blocks 2p (tile 0) and
// 2p + 1 (tile 1) of one (head, batch) and loads each key block that both
// route only once; the tensor pipe alternates between the tiles, so one
// tile's softmax runs while the other tile's MMAs execute.
//
// Schedule.  A "step" is one key block for tile 0, tile 1 or both: first every
// block both rows select (ascending), then the blocks only one row selects,
// alternating between the tiles while both have some left (ascending within a
// tile), then the rest.  Each tile therefore sees its own key blocks in the
// order "shared ascending, then its own ascending"; the online softmax makes
// the result independent of that order up to rounding.
//
// Roles (352 threads):
//   warp 10  scheduler: builds the schedule by walking the two CSR rows and
//            puts each step's (tile mask, key block) into a ring of step
//            records that runs ahead of the two consumers below;
//   warp 8   loader: TMA-loads K_s and V_{s-1} into a ring of 32 KB slots in
//            the order the MMA issuer first uses them;
//   warp 9   TMEM owner; one thread TMA-loads both Q tiles and issues every
//            MMA in one stream: per step, for each tile t in the step,
//            O_t += P_t V_{prev} (if tile t had the previous step) then
//            S_t = Q_t K_s^T; then O_t += P_t V_{prev} for the tiles of the
//            previous step that are not in this one.  Issue order keeps
//            S_t(next) after O_t += P_t V (same thread, in-order tensor pipe),
//            which is what lets P_t live in S_t's TMEM columns.
//   warps 0-3 / 4-7   softmax of tile 0 / tile 1: one query row per thread,
//            row max then exponentials in 32-column chunks (log2 domain, a
//            stabiliser that moves only past 2^8, O_t rescaled in TMEM then),
//            P_t as bf16 into the first 64 columns of S_t; at the end O_t is
//            normalised and stored (optionally to permuted rows).
// TMEM columns: S_0 [0,128), S_1 [128,256), O_0 [256,384), O_1 [384,512).
// Shared memory: Q_0, Q_1 (32 KB each), five 32 KB K/V slots, barriers.
// Every mbarrier wait is bounded (bsa::mbar_wait); on a timeout the CTA sets
// kErrWaitTimeout in the caller's error word, drains its in-flight copies and
// MMAs, frees TMEM and exits.
#include <atomic>

#include "attention_softmax.cuh"
#include "bsa_kernels.h"

namespace bsa {
namespace {

using namespace attn;

// Softmax warps per (tile, TMEM lane quarter): 1 (a thread owns a whole
// 128-column row) or 2 (column halves; the halves meet once per block to
// agree on the row max).
#ifndef BSA_PAIR_HALVES
#define BSA_PAIR_HALVES 2
#endif
constexpr int kHalves = BSA_PAIR_HALVES;
static_assert(kHalves == 1 || kHalves == 2, "one or two softmax warps per row quarter");
constexpr int kSoftWarps = 8 * kHalves;
constexpr int kColsPerThread = 128 / kHalves;
// Warpgroups: the softmax warps (tile 0, then tile 1), then one control
// warpgroup: loader, MMA issuer, scheduler and one idle warp.  At launch every
// thread has kLaunchRegs registers; the control warpgroup gives some back and
// the softmax warpgroups take them, never more than the launch total.
constexpr int kPairThreads = 32 * (kSoftWarps + 4);
constexpr int kPairProducerWarp = kSoftWarps;
constexpr int kPairMmaWarp = kSoftWarps + 1;
constexpr int kPairSchedWarp = kSoftWarps + 2;
constexpr uint32_t kLaunchRegs = kHalves == 1 ? 168 : 96;
constexpr uint32_t kSoftmaxRegs = kHalves == 1 ? 200 : 104;
constexpr uint32_t kControlRegs = kHalves == 1 ? 104 : 64;
static_assert(kSoftWarps * 32 * kSoftmaxRegs + 128 * kControlRegs <= kPairThreads * kLaunchRegs,
              "register split must stay within the launch total");
constexpr int kPairHeadDim = 128;
constexpr int kPairSlots = kHalves == 1 ? 5 : 4;
constexpr int kStepRing = 16;
constexpr uint32_t kTmemS = 0;      // + 128 * tile
constexpr uint32_t kTmemO = 256;    // + 128 * tile
// Of every 8 column pairs of a full key block, this many take their
// exponentials on the FMA pipe (exp2_poly2) instead of MUFU.
#ifndef BSA_PAIR_EMULATED_PAIRS
#define BSA_PAIR_EMULATED_PAIRS 0
#endif
constexpr int kPairEmulated = BSA_PAIR_EMULATED_PAIRS;
// Chunks of the S row kept in registers between the max and exponential
// passes (the rest are read from TMEM again).
#ifndef BSA_PAIR_KEPT_CHUNKS
#define BSA_PAIR_KEPT_CHUNKS (4 / BSA_PAIR_HALVES)
#endif
constexpr int kPairKept = BSA_PAIR_KEPT_CHUNKS;

struct PairLayout {
  static constexpr int kPanel = 128 * 128;                 // one 64-column panel: 16 KB
  static constexpr int kSlotBytes = 2 * kPanel;            // a 128 x 128 bf16 tile
  static constexpr int kQOff = 0;                          // Q_0, Q_1
  static constexpr int kRingOff = 2 * kSlotBytes;
  // Row exchange between the two halves of a row: [parity][tile][half][row]
  // floats for the row max, and the same for the block sums (dense mass).
  static constexpr int kXOff = kRingOff + kPairSlots * kSlotBytes;
  static constexpr int kXBytes = kHalves == 2 ? 2 * 2 * 2 * 2 * 128 * 4 : 0;
  static constexpr int kBarOff = kXOff + kXBytes;
  static constexpr int kBarBytes = 640;
  static constexpr int kUsed = kBarOff + kBarBytes;
};

struct PairBarriers {
  uint64_t q_full;
  uint64_t slot_full[kPairSlots];
  uint64_t slot_empty[kPairSlots];
  uint64_t step_full[kStepRing];
  uint64_t step_empty[kStepRing];
  uint64_t s_full[2];
  uint64_t p_full[2];
  uint64_t kb_full[2];
  uint64_t o_final[2];
  uint64_t drain;
  int32_t step_info[kStepRing];   // (key block << 2) | tile mask; mask 0 ends the schedule
  int32_t kb_box[2];              // key block of tile t's current S (issuer -> softmax)
  uint32_t tmem_base;
  int abort;
};

// One CSR row in global memory with its length; ids are checked on read.
struct RouteRow {
  const int32_t* ids;
  int n;
};

// Incremental walks over two ascending CSR rows a (tile 0) and b (tile 1):
// the blocks both select, and the blocks only one selects.
struct ScheduleWalker {
  RouteRow a, b;
  int k_blocks;
  int* err_word;
  int sa = 0, sb = 0;      // intersection walk
  int ua = 0, vb = 0;      // a minus b
  int ub = 0, va = 0;      // b minus a
  int last_single = 1;     // tile of the previous single step (tile 0 goes first)
  bool shared_done = false;

  __device__ int id(const RouteRow& r, int i) {
    int kb = __ldg(r.ids + i);
    if (kb < 0 || kb >= k_blocks) {
      atomicOr(err_word, kErrBadRoute);
      kb = kb < 0 ? 0 : k_blocks - 1;
    }
    return kb;
  }
  // Next block selected by both rows, or -1.
  __device__ int next_shared() {
    while (sa < a.n && sb < b.n) {
      const int x = id(a, sa), y = id(b, sb);
      if (x == y) {
        ++sa;
        ++sb;
        return x;
      }
      if (x < y) ++sa; else ++sb;
    }
    return -1;
  }
  // Next block of `r` not selected by `o` (pointers i over r, j over o).
  // This walk visits every id of r once, so it also checks that the row is
  // strictly ascending (the schedule depends on it; CSR rows from
  // bsa_route_select and bsa_pack_boolean_rows are).
  __device__ int next_unique(const RouteRow& r, const RouteRow& o, int& i, int& j, int& last) {
    while (i < r.n) {
      const int x = id(r, i++);
      if (x <= last) atomicOr(err_word, kErrBadRoute);
      last = x;
      while (j < o.n && id(o, j) < x) ++j;
      if (j >= o.n || id(o, j) != x) return x;
    }
    return -1;
  }
  int last_ua = -1, last_ub = -1;
  int pending_a = -2, pending_b = -2;   // -2: not fetched yet
  __device__ int peek_a() {
    if (pending_a == -2) pending_a = next_unique(a, b, ua, vb, last_ua);
    return pending_a;
  }
  __device__ int peek_b() {
    if (pending_b == -2) pending_b = next_unique(b, a, ub, va, last_ub);
    return pending_b;
  }
  // Next step as (key block << 2) | mask; 0 when the schedule is done.
  __device__ int next_step() {
    if (!shared_done) {
      const int x = next_shared();
      if (x >= 0) return (x << 2) | 3;
      shared_done = true;
    }
    const int xa = peek_a(), xb = peek_b();
    if (xa < 0 && xb < 0) return 0;
    const bool take_a = xb < 0 || (xa >= 0 && last_single == 1);
    if (take_a) {
      pending_a = -2;
      last_single = 0;
      return (xa << 2) | 1;
    }
    pending_b = -2;
    last_single = 1;
    return (xb << 2) | 2;
  }
};

// kTail: T is not a multiple of 128, so the last key block is partial (keys
// past T masked in the softmax, which then needs every block's id).
template <bool kDenseMass, bool kTail>
__global__ void __launch_bounds__(kPairThreads, 1)
    bsa_attention_pair_kernel(const __grid_constant__ CUtensorMap tm_q,
                              const __grid_constant__ CUtensorMap tm_k,
                              const __grid_constant__ CUtensorMap tm_v, const AttnArgs a) {
  using L = PairLayout;
  static_assert(sizeof(PairBarriers) <= L::kBarBytes, "barrier area");
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem + L::kQOff;
  uint8_t* sRing = smem + L::kRingOff;
  PairBarriers* bar = reinterpret_cast<PairBarriers*>(smem + L::kBarOff);
  volatile int* abort_flag = &bar->abort;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int qb0 = 2 * blockIdx.x;              // tile t covers query block qb0 + t
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const bool has_tile1 = qb0 + 1 < a.q_blocks;
  const int64_t rb = a.route_batch_stride ? b : 0;

  // CSR rows of both tiles; counts clamped and reported when out of range.
  auto route_of = [&](int t) -> RouteRow {
    if (t == 1 && !has_tile1) return RouteRow{nullptr, 0};
    if constexpr (kDenseMass) return RouteRow{nullptr, a.k_blocks};
    const int64_t route_row = (rb * a.heads + h) * a.q_blocks + qb0 + t;
    int n = a.counts[route_row];
    if (n < 0 || n > a.route_cols || n > a.k_blocks) {
      if (threadIdx.x == 0) atomicOr(a.err_word, kErrBadRoute);
      n = n < 0 ? 0 : min(n, min(a.route_cols, a.k_blocks));
    }
    return RouteRow{a.indices + route_row * a.route_cols, n};
  };
  const RouteRow row0 = route_of(0);
  const RouteRow row1 = route_of(1);
  const bool any_work = row0.n + row1.n > 0;
  // Softmax threads need each block's id only for a partial last block (keys
  // past T masked) or for the per-block sums of the dense-mass variant.
  constexpr bool need_kb = kDenseMass || kTail;

  if (threadIdx.x == 0) {
    uint32_t dyn_bytes;
    asm("mov.u32 %0, %%dynamic_smem_size;" : "=r"(dyn_bytes));
    const bool fits = (smem - smem_raw) + L::kUsed <= static_cast<int>(dyn_bytes);
    mbar_init(&bar->q_full, 1);
    for (int s = 0; s < kPairSlots; ++s) {
      mbar_init(&bar->slot_full[s], 1);
      mbar_init(&bar->slot_empty[s], 1);
    }
    for (int r = 0; r < kStepRing; ++r) {
      mbar_init(&bar->step_full[r], 1);
      mbar_init(&bar->step_empty[r], 2);   // the loader and the MMA issuer
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&bar->s_full[t], 1);
      mbar_init(&bar->p_full[t], 128 * kHalves);
      mbar_init(&bar->kb_full[t], 1);
      mbar_init(&bar->o_final[t], 1);
    }
    mbar_init(&bar->drain, 1);
    bar->abort = (prior_timeout(a.err_word) || !fits) ? 1 : 0;
    if (!fits) atomicOr(a.err_word, kErrSmemLayout);
    fence_mbar_init();
  }
  __syncthreads();
  if (bar->abort) return;  // uniform: set before the barrier, read after it
  if (warp == kPairMmaWarp) tmem_alloc(&bar->tmem_base, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar->tmem_base;
  // The register split sits at the top of the two role branches (not before
  // a join), so each branch is compiled against its own budget.
  if (warp >= kSoftWarps) {
   setmaxnreg_dec<kControlRegs>();
   if (warp == kPairSchedWarp) {
    // ------------------------------------------------------------ scheduler
    // Walks the two CSR rows and fills the step ring ahead of the loader and
    // the MMA issuer (both consume every step record).
    if (lane == 0 && any_work) {
      ScheduleWalker walk{row0, row1, a.k_blocks, a.err_word};
      for (int s = 0;; ++s) {
        int info;
        if constexpr (kDenseMass) {
          info = s < a.k_blocks ? ((s << 2) | (has_tile1 ? 3 : 1)) : 0;
        } else {
          info = walk.next_step();
        }
        const int r = s % kStepRing;
        if (!mbar_wait(&bar->step_empty[r], ((s / kStepRing) & 1) ^ 1, abort_flag, a.err_word))
          break;
        bar->step_info[r] = info;
        mbar_arrive(&bar->step_full[r]);
        if ((info & 3) == 0) break;
      }
    }
   } else if (warp == kPairProducerWarp) {
    // ------------------------------------------------------------ loader
    if (lane == 0 && any_work) {
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      uint32_t armed = 0, armed_phase = 0;   // per slot: load issued / its parity
      int seq = 0;
      bool ok = true;
      auto load = [&](const CUtensorMap* tm, int kb) {
        const int s = seq % kPairSlots;
        const uint32_t ph = (seq / kPairSlots) & 1;
        if (!mbar_wait(&bar->slot_empty[s], ph ^ 1, abort_flag, a.err_word)) return false;
        uint8_t* dst = sRing + s * L::kSlotBytes;
        mbar_arrive_expect_tx(&bar->slot_full[s], L::kSlotBytes);
        tma_load_4d(dst, tm, &bar->slot_full[s], 0, h, kb * 128, b);
        tma_load_4d(dst + L::kPanel, tm, &bar->slot_full[s], 64, h, kb * 128, b);
        armed |= 1u << s;
        armed_phase = (armed_phase & ~(1u << s)) | (ph << s);
        ++seq;
        return true;
      };
      int prev_mask = 0, prev_kb = 0;
      for (int s = 0; ok; ++s) {
        const int r = s % kStepRing;
        ok = mbar_wait(&bar->step_full[r], (s / kStepRing) & 1, abort_flag, a.err_word);
        if (!ok) break;
        const int info = bar->step_info[r];
        mbar_arrive(&bar->step_empty[r]);
        const int mask = info & 3;
        const int kb = info >> 2;
        // First-use order of the issuer: V of the previous step before K of
        // this one when a tile continues from the previous step.
        const bool v_first = (prev_mask & mask) != 0;
        if (prev_mask && v_first) ok = load(&tm_v, prev_kb);
        if (ok && mask) ok = load(&tm_k, kb);
        if (ok && prev_mask && !v_first) ok = load(&tm_v, prev_kb);
        if (mask == 0) break;
        prev_mask = mask;
        prev_kb = kb;
      }
      // Never leave a copy in flight into shared memory.
      int never = 0;
#pragma unroll
      for (int s = 0; s < kPairSlots; ++s)
        if (armed & (1u << s))
          mbar_wait(&bar->slot_full[s], (armed_phase >> s) & 1u, &never, a.err_word);
    }
   } else if (warp == kPairMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && any_work) {
      const uint32_t idesc_s = idesc_bf16_f32(128, 128, false);
      const uint32_t idesc_o = idesc_bf16_f32(128, kPairHeadDim, true);
      const uint32_t ring_addr = smem_u32(sRing);
      const uint64_t kdesc0 = sdesc_sw128(ring_addr, 16, 1024);
      const uint64_t vdesc0 = sdesc_sw128(ring_addr, L::kPanel, 1024);
      const uint64_t qdesc0 = sdesc_sw128(smem_u32(sQ), 16, 1024);
      tma_prefetch_desc(&tm_q);
      mbar_arrive_expect_tx(&bar->q_full, (has_tile1 ? 2 : 1) * L::kSlotBytes);
      for (int t = 0; t < (has_tile1 ? 2 : 1); ++t) {
        uint8_t* dq = sQ + t * L::kSlotBytes;
        tma_load_4d(dq, &tm_q, &bar->q_full, 0, h, (qb0 + t) * 128, b);
        tma_load_4d(dq + L::kPanel, &tm_q, &bar->q_full, 64, h, (qb0 + t) * 128, b);
      }
      bool ok = mbar_wait(&bar->q_full, 0, abort_flag, a.err_word);
      int seq = 0;
      int prev_mask = 0;
      int pv0 = 0, pv1 = 0;      // PV issued per tile
      auto issue_pv = [&](int t, int vslot) {
        // O_t += P_t V: P (bf16) in S_t's first 64 columns, V from the slot.
        const int j = t ? pv1 : pv0;
        if (!mbar_wait(&bar->p_full[t], j & 1, abort_flag, a.err_word)) return false;
        tc_fence_after();
        const uint64_t vd = vdesc0 + static_cast<uint64_t>((vslot * L::kSlotBytes) >> 4);
        const uint32_t pa = tmem + kTmemS + t * 128;
        const uint32_t d = tmem + kTmemO + t * 128;
#pragma unroll
        for (int kk = 0; kk < 128 / 16; ++kk)
          umma_bf16_ts(d, pa + kk * 8, vd + static_cast<uint64_t>((kk * 16 * 128) >> 4), idesc_o,
                       (j > 0 || kk > 0) ? 1u : 0u);
        if (t) ++pv1; else ++pv0;
        if (j + 1 == (t ? row1.n : row0.n)) umma_commit(&bar->o_final[t]);
        return true;
      };
      for (int s = 0; ok; ++s) {
        const int r = s % kStepRing;
        ok = mbar_wait(&bar->step_full[r], (s / kStepRing) & 1, abort_flag, a.err_word);
        if (!ok) break;
        const int info = bar->step_info[r];
        mbar_arrive(&bar->step_empty[r]);
        const int mask = info & 3;
        const int kb = info >> 2;
        const bool v_first = (prev_mask & mask) != 0;
        int vslot = -1, vphase = 0, kslot = -1, kphase = 0;
        if (prev_mask && v_first) { vslot = seq % kPairSlots; vphase = (seq / kPairSlots) & 1; ++seq; }
        if (mask) { kslot = seq % kPairSlots; kphase = (seq / kPairSlots) & 1; ++seq; }
        if (prev_mask && !v_first) { vslot = seq % kPairSlots; vphase = (seq / kPairSlots) & 1; ++seq; }
        bool v_ready = false, k_ready = false;
        for (int t = 0; ok && t < 2; ++t) {
          if (!((mask >> t) & 1)) continue;
          if ((prev_mask >> t) & 1) {
            if (!v_ready) ok = v_ready = mbar_wait(&bar->slot_full[vslot], vphase, abort_flag, a.err_word);
            if (ok) ok = issue_pv(t, vslot);
            if (!ok) break;
          }
          if (!k_ready) ok = k_ready = mbar_wait(&bar->slot_full[kslot], kphase, abort_flag, a.err_word);
          if (!ok) break;
          if (need_kb) {
            bar->kb_box[t] = kb;
            mbar_arrive(&bar->kb_full[t]);
          }
          tc_fence_after();
          const uint64_t kd = kdesc0 + static_cast<uint64_t>((kslot * L::kSlotBytes) >> 4);
          const uint64_t qd = qdesc0 + static_cast<uint64_t>((t * L::kSlotBytes) >> 4);
          const uint32_t d = tmem + kTmemS + t * 128;
#pragma unroll
          for (int kk = 0; kk < kPairHeadDim / 16; ++kk) {
            const uint64_t off = static_cast<uint64_t>(((kk >> 2) * L::kPanel + (kk & 3) * 32) >> 4);
            umma_bf16_ss(d, qd + off, kd + off, idesc_s, kk > 0 ? 1u : 0u);
          }
          umma_commit(&bar->s_full[t]);
        }
        if (!ok) break;
        if (mask) umma_commit(&bar->slot_empty[kslot]);
        // Tiles of the previous step that skip this one: their PV now.
        for (int t = 0; ok && t < 2; ++t) {
          if (!((prev_mask >> t) & 1) || ((mask >> t) & 1)) continue;
          if (!v_ready) ok = v_ready = mbar_wait(&bar->slot_full[vslot], vphase, abort_flag, a.err_word);
          if (ok) ok = issue_pv(t, vslot);
        }
        if (!ok) break;
        if (prev_mask) umma_commit(&bar->slot_empty[vslot]);
        if (mask == 0) break;
        prev_mask = mask;
      }
      int never = 0;
      umma_commit(&bar->drain);
      mbar_wait(&bar->drain, 0, &never, a.err_word);
    }
   }
  } else {
    setmaxnreg_inc<kSoftmaxRegs>();
    // ------------------------------------------------------------ softmax
    const int t = warp / (4 * kHalves);        // tile
    const int wq = warp & 3;                   // TMEM lane quarter
    const int hf = (warp / 4) % kHalves;       // column half of the row (kHalves == 2)
    const int row = wq * 32 + lane;            // query row == TMEM lane
    const uint32_t lane_addr = static_cast<uint32_t>(wq * 32) << 16;
    const int qb = qb0 + t;
    const int64_t token = static_cast<int64_t>(qb) * 128 + row;
    const int n = t ? row1.n : row0.n;
    const bool row_valid = (t == 0 || has_tile1) && token < a.tokens;
    // This thread's S columns, its P columns (bf16 pairs, half as many) and
    // its O columns.
    const uint32_t sbuf = tmem + lane_addr + kTmemS + t * 128 + hf * kColsPerThread;
    const uint32_t pbuf = tmem + lane_addr + kTmemS + t * 128 + hf * (kColsPerThread / 2);
    const uint32_t obuf = tmem + lane_addr + kTmemO + t * 128 + hf * kColsPerThread;
    float* xmax = reinterpret_cast<float*>(smem + L::kXOff);            // [2][2][2][128]
    float* xsum = xmax + 2 * 2 * 2 * 128;
    auto xidx = [&](int parity, int half) { return ((parity * 2 + t) * 2 + half) * 128 + row; };
    const uint32_t pair_bar = 1 + t * 4 + wq;  // named barrier of the row's two halves
    const float c = a.scale * kLog2e;
    const float2 c2 = make_float2(c, c);
    float m_run = -INFINITY;   // stabiliser (log2 units) the row's O and l are relative to
    float l = 0.f;             // this thread's part of the row sum, relative to m_run
    bool ok = true;
    for (int j = 0; ok && j < n; ++j) {
      int kb = 0;
      if (need_kb) {
        ok = mbar_wait(&bar->kb_full[t], j & 1, abort_flag, a.err_word);
        if (!ok) break;
        kb = bar->kb_box[t];
      }
      ok = mbar_wait(&bar->s_full[t], j & 1, abort_flag, a.err_word);
      if (!ok) break;
      tc_fence_after();
      const int64_t valid = a.tokens - static_cast<int64_t>(kb) * 128 - hf * kColsPerThread;
      const bool partial = kTail && valid < kColsPerThread;
      uint32_t keep[kPairKept][32];
      float mrow = row_max<kColsPerThread, kPairKept>(sbuf, partial, valid, keep) * c;
      if constexpr (kHalves == 2) {
        // Both halves' S columns are in registers now, so P may overwrite
        // them after this barrier; the row max is the larger half's.
        xmax[xidx(j & 1, hf)] = mrow;
        named_bar_sync(pair_bar, 64);
        mrow = fmaxf(mrow, xmax[xidx(j & 1, hf ^ 1)]);
      }
      const bool need = mrow > m_run + kRescaleThreshold;
      const float m_used = need ? mrow : m_run;
      const float2 neg_m = make_float2(-m_used, -m_used);
      // With a partial block possible, every exponential stays on MUFU (one
      // code path for masked and full blocks).
      const float2 rs = row_exp<kColsPerThread, kTail ? 0 : kPairEmulated, kPairKept>(
          sbuf, partial, valid, c2, neg_m, keep, pbuf);
      // O_t holds the blocks before j relative to m_run; it is complete here
      // (its last PV was issued before this S, and s_full tracks both), and
      // PV of block j waits for p_full below.
      if (j > 0 && __any_sync(0xffffffffu, need)) {
        const float o_scale = need ? ex2_approx(m_run - m_used) : 1.f;
#pragma unroll 1
        for (int cc = 0; cc < kColsPerThread / 32; ++cc) {
          uint32_t o[32];
          tmem_ld_32x32b_x32(obuf + cc * 32, o);
          tmem_wait_ld();
          reg_fence<32>(o);
#pragma unroll
          for (int x = 0; x < 32; ++x) o[x] = __float_as_uint(__uint_as_float(o[x]) * o_scale);
          tmem_st_32x32b_x32(obuf + cc * 32, o);
        }
      }
      l = l * ex2_approx(m_run - m_used) + (rs.x + rs.y);   // m_run = -inf at j = 0: l = 0
      m_run = m_used;
      if constexpr (kDenseMass) {
        float block_sum = rs.x + rs.y;
        if constexpr (kHalves == 2) {
          xsum[xidx(j & 1, hf)] = block_sum;
          named_bar_sync(pair_bar, 64);
          block_sum = xsum[xidx(j & 1, 0)] + xsum[xidx(j & 1, 1)];
        }
        if (row_valid && hf == 0) {
          float* dst = a.block_lse + static_cast<int64_t>(kb) * a.tokens + token;
          dst[(static_cast<int64_t>(b) * a.heads + h) * a.k_blocks * a.tokens] =
              m_used + __log2f(block_sum);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bar->p_full[t]);
    }
    // ---------------------------------------------------------- epilogue
    if constexpr (kHalves == 2) {
      // Both halves used the same stabilisers: the row sum is the sum of parts.
      named_bar_sync(pair_bar, 64);
      xsum[xidx(0, hf)] = l;
      named_bar_sync(pair_bar, 64);
      l = xsum[xidx(0, 0)] + xsum[xidx(0, 1)];
    }
    if (ok && n > 0) {
      ok = mbar_wait(&bar->o_final[t], 0, abort_flag, a.err_word);
      tc_fence_after();
    }
    int64_t out_token = token;
    bool row_store = row_valid;
    if (a.out_rows != nullptr && row_valid) {
      out_token = __ldg(a.out_rows + token);
      if (out_token < 0 || out_token >= a.tokens) {
        atomicOr(a.err_word, kErrBadRoute);
        row_store = false;
      }
    }
    const float inv_l = (n > 0 && l > 0.f) ? 1.f / l : 0.f;
    __nv_bfloat16* out = a.out + b * a.out_stride_b + out_token * a.out_stride_t +
                         h * a.out_stride_h + hf * kColsPerThread;
#pragma unroll 1
    for (int cc = 0; cc < kColsPerThread / 32; ++cc) {
      uint32_t o[32];
      if (ok && n > 0) {
        tmem_ld_32x32b_x32(obuf + cc * 32, o);
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
    if (row_valid && hf == 0 && a.lse != nullptr) {
      a.lse[(static_cast<int64_t>(b) * a.heads + h) * a.tokens + token] =
          (n > 0 && l > 0.f) ? (m_run + __log2f(l)) * kLn2 : -INFINITY;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kPairMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <bool kDenseMass, bool kTail>
cudaError_t launch_pair_impl(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                             const AttnArgs& a, cudaStream_t stream) {
  using L = PairLayout;
  static std::atomic<int> smem_bytes[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  int bytes = (dev >= 0 && dev < 64) ? smem_bytes[dev].load(std::memory_order_acquire) : 0;
  if (bytes == 0) {
    int optin = 0;
    e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e != cudaSuccess) return e;
    // The layout needs kUsed bytes from a 1024-byte-aligned base.
    bytes = optin < L::kUsed + 1024 ? optin : L::kUsed + 1024;
    if (bytes < L::kUsed) return cudaErrorInvalidConfiguration;
    // The register split inside the kernel assumes exactly kLaunchRegs per
    // thread at launch; anything else could leave an increase waiting.
    cudaFuncAttributes attr{};
    e = cudaFuncGetAttributes(&attr, bsa_attention_pair_kernel<kDenseMass, kTail>);
    if (e != cudaSuccess) return e;
    if (attr.numRegs != static_cast<int>(kLaunchRegs)) return cudaErrorInvalidConfiguration;
    e = cudaFuncSetAttribute(bsa_attention_pair_kernel<kDenseMass, kTail>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) smem_bytes[dev].store(bytes, std::memory_order_release);
  }
  const dim3 grid(static_cast<unsigned>((a.q_blocks + 1) / 2), static_cast<unsigned>(a.heads),
                  static_cast<unsigned>(a.batch));
  bsa_attention_pair_kernel<kDenseMass, kTail><<<grid, kPairThreads, bytes, stream>>>(tq, tk, tv,
                                                                                     a);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_attention_pair(const CUtensorMap& tq, const CUtensorMap& tk,
                                  const CUtensorMap& tv, const AttnArgs& a, cudaStream_t stream) {
  if (a.block != 128) return cudaErrorInvalidValue;
  if (a.batch == 0 || a.heads == 0 || a.q_blocks == 0) return cudaSuccess;
  const bool tail = (a.tokens % 128) != 0;
  if (a.block_lse != nullptr)
    return tail ? launch_pair_impl<true, true>(tq, tk, tv, a, stream)
                : launch_pair_impl<true, false>(tq, tk, tv, a, stream);
  return tail ? launch_pair_impl<false, true>(tq, tk, tv, a, stream)
              : launch_pair_impl<false, false>(tq, tk, tv, a, stream);
}

}  // namespace bsa
