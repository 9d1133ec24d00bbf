// (b) Sampled block mass on tcgen05.
//
// Reference semantics: attention_backends/flex.py:205-251.  For every head,
// the sampled queries ([Qb*S, D], S evenly spaced tokens per block) attend to
// all sampled keys ([Qb*S, D]) with an additive per-key weight
// log(block_size / S); the softmax row is then summed over the S key samples of
// each key block and averaged over the S query samples of each query block:
//   mass[h, qb, kb] = (1/S) * sum_{r in qb} sum_{k in kb} softmax_r(k).
// With round_bf16 set, scores are rounded like the reference's bf16 matmul
// output and bf16 `* score_scale` (flex.py:245) before the fp32 softmax.
//
// One CTA per (128 sampled query rows, head, batch).  The 128-key tiles of the
// sampled keys stream twice through a TMA ring: pass 1 computes every row's
// log-sum-exp, pass 2 the normalised per-block sums (S consecutive rows of a
// query block are S consecutive lanes, reduced with shuffles).
//   warp 4 TMA producer, warp 5 TMEM allocator + tcgen05.mma issuer,
//   warps 0-3 softmax / reduction (thread i owns sampled row i).
#include "bsa_kernels.h"

namespace bsa {
namespace {

constexpr int kMassThreads = 192;
constexpr int kSlots = 5;
constexpr int kTile = 128;
constexpr float kLog2eM = 1.4426950408889634f;
constexpr int kQBytes = kTile * 256;
constexpr int kSlotBytes = kTile * 256;
constexpr int kPanel = kTile * 128;
constexpr int kRingOff = kQBytes;
constexpr int kBiasOff = kRingOff + kSlots * kSlotBytes;
constexpr int kMaxBlocks = 4096;
constexpr int kBarOff = kBiasOff + kMaxBlocks * 4;
constexpr int kMassSmem = kBarOff + 256 + 1024;

struct MassBarriers {
  uint64_t q_full;
  uint64_t s_full[2];
  uint64_t s_free[2];
  uint64_t drain;
  uint64_t slot_full[kSlots];
  uint64_t slot_empty[kSlots];
  uint32_t tmem_base;
  int abort;
};

template <int LOG2S>
__global__ void __launch_bounds__(kMassThreads, 1)
    sampled_mass_kernel(const __grid_constant__ CUtensorMap tm_q,
                        const __grid_constant__ CUtensorMap tm_k, const MassArgs a) {
  constexpr int S = 1 << LOG2S;
  constexpr int kGroups = kTile / S;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem;
  uint8_t* sRing = smem + kRingOff;
  float* sBias = reinterpret_cast<float*>(smem + kBiasOff);
  __shared__ float sRed[8];
  MassBarriers* bar = reinterpret_cast<MassBarriers*>(smem + kBarOff);
  volatile int* abort_flag = &bar->abort;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int qt = blockIdx.x;
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int n_tiles = static_cast<int>((a.n_rows + kTile - 1) / kTile);
  const int steps = 2 * n_tiles;

  if (threadIdx.x == 0) {
    mbar_init(&bar->q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar->s_full[i], 1);
      mbar_init(&bar->s_free[i], 128);
    }
    mbar_init(&bar->drain, 1);
    for (int s = 0; s < kSlots; ++s) {
      mbar_init(&bar->slot_full[s], 1);
      mbar_init(&bar->slot_empty[s], 1);
    }
    bar->abort = prior_timeout(a.err_word) ? 1 : 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (bar->abort) return;  // uniform: set before the barrier, read after it
  for (int i = threadIdx.x; i < a.q_blocks; i += kMassThreads)
    sBias[i] = a.block_bias != nullptr ? a.block_bias[i] : 0.f;
  if (warp == 5) tmem_alloc(&bar->tmem_base, 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar->tmem_base;

  if (warp == 4) {
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      mbar_arrive_expect_tx(&bar->q_full, kQBytes);
      tma_load_4d(sQ, &tm_q, &bar->q_full, 0, h, qt * kTile, b);
      tma_load_4d(sQ + kPanel, &tm_q, &bar->q_full, 64, h, qt * kTile, b);
      uint32_t armed[kSlots];
      for (int s = 0; s < kSlots; ++s) armed[s] = 2;
      for (int i = 0; i < steps; ++i) {
        const int s = i % kSlots;
        const uint32_t ph = (i / kSlots) & 1;
        if (!mbar_wait(&bar->slot_empty[s], ph ^ 1, abort_flag, a.err_word)) break;
        const int kt = i % n_tiles;
        uint8_t* dst = sRing + s * kSlotBytes;
        mbar_arrive_expect_tx(&bar->slot_full[s], kSlotBytes);
        tma_load_4d(dst, &tm_k, &bar->slot_full[s], 0, h, kt * kTile, b);
        tma_load_4d(dst + kPanel, &tm_k, &bar->slot_full[s], 64, h, kt * kTile, b);
        armed[s] = ph;
      }
      int never = 0;
      mbar_wait(&bar->q_full, 0, &never, a.err_word);
      for (int s = 0; s < kSlots; ++s)
        if (armed[s] < 2) mbar_wait(&bar->slot_full[s], armed[s], &never, a.err_word);
    }
  } else if (warp == 5) {
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(128, kTile, false);
      const uint32_t q_addr = smem_u32(sQ);
      const uint32_t ring_addr = smem_u32(sRing);
      bool ok = mbar_wait(&bar->q_full, 0, abort_flag, a.err_word);
      for (int i = 0; ok && i < steps; ++i) {
        const int s = i % kSlots;
        ok = mbar_wait(&bar->slot_full[s], (i / kSlots) & 1, abort_flag, a.err_word);
        if (ok && i >= 2) ok = mbar_wait(&bar->s_free[i & 1], ((i >> 1) - 1) & 1, abort_flag, a.err_word);
        if (!ok) break;
        tc_fence_after();
        const uint32_t k_addr = ring_addr + s * kSlotBytes;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (kk & 3) * 32;
          const uint64_t da = sdesc_sw128(q_addr + (kk >> 2) * kPanel + off, 16, 1024);
          const uint64_t db = sdesc_sw128(k_addr + (kk >> 2) * kPanel + off, 16, 1024);
          umma_bf16_ss(tmem + (i & 1) * 128, da, db, idesc, kk > 0 ? 1u : 0u);
        }
        umma_commit(&bar->s_full[i & 1]);
        umma_commit(&bar->slot_empty[s]);
      }
      int never = 0;
      umma_commit(&bar->drain);
      mbar_wait(&bar->drain, 0, &never, a.err_word);
    }
  } else {
    const int row = threadIdx.x;
    const uint32_t lane_addr = static_cast<uint32_t>(warp * 32) << 16;
    const int64_t qrow = static_cast<int64_t>(qt) * kTile + row;
    float m2 = -INFINITY, l = 0.f, inv_l = 0.f;
    bool ok = true;
    for (int i = 0; i < steps; ++i) {
      ok = mbar_wait(&bar->s_full[i & 1], (i >> 1) & 1, abort_flag, a.err_word);
      if (!ok) break;
      tc_fence_after();
      float y[kTile];
      uint32_t r[kTile];
#pragma unroll
      for (int cc = 0; cc < kTile / 32; ++cc)
        tmem_ld_32x32b_x32(tmem + lane_addr + (i & 1) * 128 + cc * 32, r + cc * 32);
      tmem_wait_ld();
      reg_fence<kTile>(r);
#pragma unroll
      for (int x = 0; x < kTile; ++x) y[x] = __uint_as_float(r[x]);
      tc_fence_before();
      mbar_arrive(&bar->s_free[i & 1]);
      const int kt = i % n_tiles;
      const int64_t key0 = static_cast<int64_t>(kt) * kTile;
#pragma unroll
      for (int x = 0; x < kTile; ++x) {
        float sc = y[x];
        if (a.round_bf16) sc = round_to_bf16(round_to_bf16(sc) * a.scale);
        else sc = sc * a.scale;
        const int64_t key = key0 + x;
        y[x] = key < a.n_rows ? (sc + sBias[key >> LOG2S]) * kLog2eM : -INFINITY;
      }
      if (i < n_tiles) {
        float mx = y[0];
#pragma unroll
        for (int x = 1; x < kTile; ++x) mx = fmaxf(mx, y[x]);
        const float m_new = fmaxf(m2, mx);
        float rs = 0.f;
#pragma unroll
        for (int x = 0; x < kTile; ++x) rs += ex2_approx(y[x] - m_new);
        l = l * ex2_approx(m2 - m_new) + rs;
        m2 = m_new;
        if (i == n_tiles - 1) inv_l = 1.f / l;
      } else {
        float g[kGroups];
#pragma unroll
        for (int gi = 0; gi < kGroups; ++gi) {
          float acc = 0.f;
#pragma unroll
          for (int x = 0; x < S; ++x) acc += ex2_approx(y[gi * S + x] - m2);
          g[gi] = qrow < a.n_rows ? acc * inv_l : 0.f;
        }
        if constexpr (S > 1) {
#pragma unroll
          for (int gi = 0; gi < kGroups; ++gi) {
#pragma unroll
            for (int off = 1; off < (S < 32 ? S : 32); off <<= 1)
              g[gi] += __shfl_xor_sync(0xffffffffu, g[gi], off);
          }
        }
        const int64_t kb0 = key0 >> LOG2S;
        const int64_t out_rows = (static_cast<int64_t>(b) * a.heads + h) * a.q_blocks;
        if constexpr (S <= 32) {
          const int64_t qblock = qrow >> LOG2S;
          if ((row & (S - 1)) == 0 && qblock < a.q_blocks) {
            float* dst = a.mass + (out_rows + qblock) * a.q_blocks;
#pragma unroll
            for (int gi = 0; gi < kGroups; ++gi)
              if (kb0 + gi < a.q_blocks) dst[kb0 + gi] = g[gi] * a.mass_scale;
          }
        } else {
          // A query block spans S/32 warps: combine the warp sums in shared
          // memory (softmax warps only, named barrier 1).
          if (lane == 0)
#pragma unroll
            for (int gi = 0; gi < kGroups; ++gi) sRed[warp * kGroups + gi] = g[gi];
          asm volatile("bar.sync 1, 128;" ::: "memory");
          constexpr int kWarpsPerBlock = S / 32;
          if (row < (4 / kWarpsPerBlock) * kGroups) {
            const int qsub = row / kGroups;
            const int gi = row % kGroups;
            float acc = 0.f;
            for (int w = 0; w < kWarpsPerBlock; ++w) acc += sRed[(qsub * kWarpsPerBlock + w) * kGroups + gi];
            const int64_t qblock = (static_cast<int64_t>(qt) * kTile >> LOG2S) + qsub;
            if (qblock < a.q_blocks && kb0 + gi < a.q_blocks)
              a.mass[(out_rows + qblock) * a.q_blocks + kb0 + gi] = acc * a.mass_scale;
          }
          asm volatile("bar.sync 1, 128;" ::: "memory");
        }
      }
    }
    (void)ok;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

template <int LOG2S>
cudaError_t launch_log2s(const CUtensorMap& tq, const CUtensorMap& tk, const MassArgs& a,
                         cudaStream_t stream) {
  static bool configured[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    e = cudaFuncSetAttribute(sampled_mass_kernel<LOG2S>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, kMassSmem);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  const dim3 grid(static_cast<unsigned>((a.n_rows + kTile - 1) / kTile),
                  static_cast<unsigned>(a.heads), static_cast<unsigned>(a.batch));
  sampled_mass_kernel<LOG2S><<<grid, kMassThreads, kMassSmem, stream>>>(tq, tk, a);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_sampled_mass(const CUtensorMap& tq, const CUtensorMap& tk, const MassArgs& a,
                                cudaStream_t stream) {
  if (a.batch == 0 || a.heads == 0 || a.n_rows == 0) return cudaSuccess;
  if (a.q_blocks > kMaxBlocks) return cudaErrorInvalidValue;
  switch (a.samples) {
    case 1: return launch_log2s<0>(tq, tk, a, stream);
    case 2: return launch_log2s<1>(tq, tk, a, stream);
    case 4: return launch_log2s<2>(tq, tk, a, stream);
    case 8: return launch_log2s<3>(tq, tk, a, stream);
    case 16: return launch_log2s<4>(tq, tk, a, stream);
    case 32: return launch_log2s<5>(tq, tk, a, stream);
    case 64: return launch_log2s<6>(tq, tk, a, stream);
    case 128: return launch_log2s<7>(tq, tk, a, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace bsa
