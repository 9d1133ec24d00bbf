// Shared device helpers for the sm_100a kernels of the routed block-sparse
// attention path: mbarriers with bounded waits, TMA tile loads (no multicast),
// tcgen05 MMA / TMEM access and the UMMA shared-memory and instruction
// descriptors.  Everything here is written against the public PTX ISA.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace bsa {

// ---------------------------------------------------------------------------
// Error words written by kernels (bitwise OR into a caller-provided int32).
// ---------------------------------------------------------------------------
enum DeviceError : int {
  kErrWaitTimeout = 1 << 0,   // an mbarrier wait exceeded its time limit
  kErrBadRoute = 1 << 1,      // a CSR count/index was out of range (skipped)
  kErrTmemAlloc = 1 << 2,     // TMEM allocation returned an unexpected address
  kErrSmemLayout = 1 << 3,    // the dynamic shared memory cannot hold the kernel's layout
};

// A wait on an mbarrier gives up after this many nanoseconds; the kernel then
// sets kErrWaitTimeout, raises the CTA-wide abort flag and drains.
constexpr uint64_t kWaitTimeoutNs = 2000ull * 1000ull * 1000ull;  // 2 s
constexpr uint32_t kWaitMaxPolls = 1u << 28;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ bool elect_one_lane() {
  return (threadIdx.x & 31) == 0;
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Non-blocking test of the phase with the given parity (try_wait may suspend
// the thread for a while; a thread that polls several barriers must not).
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity, giving up after
// ``timeout_ns`` of %globaltimer (or kWaitMaxPolls polls).  Returns false when
// the CTA is aborting (flag set by any thread) or the wait timed out, in which
// case the abort flag and the caller's error word are set.
__device__ __forceinline__ bool mbar_wait_for(uint64_t* bar, uint32_t parity,
                                              volatile int* abort_flag, int* err_word,
                                              uint64_t timeout_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_timer_ns();
  for (uint32_t poll = 1; poll < kWaitMaxPolls; ++poll) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if ((poll & 63) == 0) {
      // Another CTA of this launch (or an earlier one) already timed out.
      if (err_word && (*reinterpret_cast<volatile int*>(err_word) & kErrWaitTimeout)) {
        *abort_flag = 1;
        return false;
      }
      if (global_timer_ns() - start > timeout_ns) break;
    }
  }
  *abort_flag = 1;
  if (err_word) atomicOr(err_word, kErrWaitTimeout);
  return false;
}

// The kernels' wait: mbar_wait_for with the library-wide limit kWaitTimeoutNs.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          volatile int* abort_flag, int* err_word) {
  return mbar_wait_for(bar, parity, abort_flag, err_word, kWaitTimeoutNs);
}

// True when an earlier timeout was recorded in the error word: kernels then
// skip their work so a systemic failure ends quickly instead of timing out
// CTA by CTA.  Cleared by the host when it reads the word.
__device__ __forceinline__ bool prior_timeout(const int* err_word) {
  return err_word && (*reinterpret_cast<const volatile int*>(err_word) & kErrWaitTimeout);
}

// ---------------------------------------------------------------------------
// Register reallocation between warpgroups (setmaxnreg): all four warps of a
// warpgroup execute the same instruction.  The block's registers at launch
// (threads x registers per thread) must cover every warpgroup's new share, or
// an increase waits for registers that never come: callers check the
// kernel's register count on the host before launching.
// ---------------------------------------------------------------------------
template <uint32_t kRegs>
__device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegs));
}
template <uint32_t kRegs>
__device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegs));
}

// ---------------------------------------------------------------------------
// TMA (cp.async.bulk.tensor), CTA-local destination, no multicast.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3),
      "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: TMEM allocation, MMA, commit, loads/stores, fences.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (bf16 inputs, fp32 accumulate).
__device__ __forceinline__ void umma_bf16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]^T, kind::f16.  A (M=128 rows x K=16) lives
// in TMEM: row m in lane m, K pairs packed low/high in consecutive 32-bit
// columns (8 columns per K=16 step).
__device__ __forceinline__ void umma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive (once) on an mbarrier when all previously issued tcgen05.mma of this
// thread have completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Registers written by tcgen05.ld are valid only after tcgen05.wait::ld.  The
// empty asm makes every later use depend on a definition placed after the
// wait, so the compiler cannot hoist a use above it.
template <int N>
__device__ __forceinline__ void reg_fence(uint32_t* r) {
#pragma unroll
  for (int i = 0; i < N; ++i) asm volatile("" : "+r"(r[i]));
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp receives
// lane (warp_lane_base + i), columns [col, col + 32).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// One 32-bit column: thread i of the warp writes lane (warp_lane_base + i).
__device__ __forceinline__ void tmem_st_32x32b_x1(uint32_t taddr, uint32_t r) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};" ::"r"(taddr), "r"(r) : "memory");
}

__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}

// ---------------------------------------------------------------------------
// UMMA descriptors.
// ---------------------------------------------------------------------------
// Instruction descriptor, kind::f16: bf16 A/B, fp32 D, dense.
//   [4,6) D format (1 = f32), [7,10) A format (1 = bf16), [10,13) B format,
//   [15] A major (0 = K), [16] B major (0 = K, 1 = MN), [17,23) N>>3, [24,29) M>>4.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(uint32_t m, uint32_t n, bool b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((b_mn_major ? 1u : 0u) << 16) |
         ((n >> 3) << 17) | ((m >> 4) << 24);
}

// Shared-memory matrix descriptor for a 128-byte-swizzled canonical layout.
//   [0,14) start>>4, [16,30) leading byte offset>>4, [32,46) stride byte
//   offset>>4, [46,48) version (1 on sm_100), [61,64) layout (2 = SWIZZLE_128B).
// K-major operands: rows of 128 B (64 bf16 of K), 8-row atoms 1024 B apart
// (SBO = 1024); LBO is unused.  MN-major operands: 64 contiguous MN elements
// per 128-B row, LBO = byte distance between 64-element MN panels, SBO = byte
// distance between 8-row K groups (1024).
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr, uint32_t lbo_bytes,
                                                uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// Byte offset of the 16-byte chunk `chunk` (0..7) of row `row` inside a
// 128-byte-swizzled panel whose rows are 128 bytes.
__device__ __forceinline__ uint32_t sw128_offset(uint32_t row, uint32_t chunk) {
  return row * 128u + (((chunk ^ (row & 7u)) & 7u) << 4);
}

// ---------------------------------------------------------------------------
// Math helpers.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// 2^x for a pair of values on the FMA pipe (no MUFU), used for a share of the
// softmax exponentials so the MUFU pipe is not the bottleneck.
// Method: Cody-Waite split x = n + f with n = rint(x) (the 1.5*2^23 rounding
// constant), f in [-1/2, 1/2]; 2^f by a degree-3 polynomial whose
// coefficients were fitted for this kernel with the Remez exchange algorithm
// (minimax relative error 7.5e-5 on [-1/2, 1/2], far below the 2^-8 rounding
// of the bf16 probabilities; fit_exp2_poly.py next to this file derives them);
// 2^n is added to the exponent bits.  Inputs are
// clamped to >= -126, so results below 2^-126 come out as ~2^-126 instead of 0.
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
  x.x = fmaxf(x.x, -126.0f);
  x.y = fmaxf(x.y, -126.0f);
  const float2 t = __fadd2_rn(x, make_float2(kRound, kRound));
  const float2 n = __fadd2_rn(t, make_float2(-kRound, -kRound));
  const float2 f = __ffma2_rn(n, make_float2(-1.0f, -1.0f), x);
  float2 p = __ffma2_rn(f, make_float2(0.0551716685f, 0.0551716685f),
                        make_float2(0.2426111251f, 0.2426111251f));
  p = __ffma2_rn(p, f, make_float2(0.6932609677f, 0.6932609677f));
  p = __ffma2_rn(p, f, make_float2(0.9999280572f, 0.9999280572f));
  const uint32_t b0 = __float_as_uint(p.x) + (__float_as_uint(t.x) << 23);
  const uint32_t b1 = __float_as_uint(p.y) + (__float_as_uint(t.y) << 23);
  return make_float2(__uint_as_float(b0), __uint_as_float(b1));
}

// bf16 round-to-nearest-even of two floats without the conversion unit:
// t = x * (2^16 + 1), hi = t - (t - x) keeps the 8 leading significand bits
// with ties to even (Veltkamp splitting; exact for |x| < 2^111).  Explicit _rn
// operations: a fused multiply-add would break it.
__device__ __forceinline__ float2 round2_bf16(float2 x) {
  const float2 t = __fmul2_rn(x, make_float2(65537.f, 65537.f));
  const float2 d = __ffma2_rn(x, make_float2(-1.f, -1.f), t);
  return __ffma2_rn(d, make_float2(-1.f, -1.f), t);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ float round_to_bf16(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

}  // namespace bsa
