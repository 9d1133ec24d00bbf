// Test-only diagnostics built into tests/diag/libbsa_diag.so (never linked
// into libbsa.so).  They run the product's own device helpers from
// bsa_common.cuh in isolation so that tests can check them directly:
//   * bsa_diag_exp2: element-wise 2^x through the two exponential paths the
//     softmax kernels use (MUFU ex2.approx and the exp2_poly2 polynomial);
//   * bsa_diag_unarmed_wait: one bounded mbarrier wait on a barrier that
//     nothing arrives on, with a caller-chosen short limit, so a test can see
//     the timeout path report kErrWaitTimeout and return (no trap, no fault,
//     no unbounded wait).
#include <stdint.h>

#include "bsa_common.cuh"

namespace {

__global__ void exp2_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t n,
                            int mode) {
  const int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 2;
  if (i >= n) return;
  const float x0 = x[i];
  const float x1 = i + 1 < n ? x[i + 1] : 0.f;
  float2 r;
  if (mode == 1) {
    r = bsa::exp2_poly2(make_float2(x0, x1));
  } else {
    r = make_float2(bsa::ex2_approx(x0), bsa::ex2_approx(x1));
  }
  y[i] = r.x;
  if (i + 1 < n) y[i + 1] = r.y;
}

// One warp.  Lane 0 initialises an mbarrier that expects one arrival, which
// never comes, and waits on phase 0 with the product's bounded wait.  The
// result records whether the wait returned true, the nanoseconds it took and
// the CTA's abort flag afterwards.
__global__ void unarmed_wait_kernel(uint64_t timeout_ns, int* err_word,
                                    long long* result) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    abort_flag = 0;
    bsa::mbar_init(&bar, 1);
    bsa::fence_mbar_init();
  }
  __syncwarp();
  if (threadIdx.x == 0) {
    const uint64_t t0 = bsa::global_timer_ns();
    const bool done = bsa::mbar_wait_for(&bar, 0, &abort_flag, err_word, timeout_ns);
    const uint64_t t1 = bsa::global_timer_ns();
    result[0] = done ? 1 : 0;
    result[1] = static_cast<long long>(t1 - t0);
    result[2] = abort_flag;
    asm volatile("mbarrier.inval.shared::cta.b64 [%0];" ::"r"(bsa::smem_u32(&bar)) : "memory");
  }
}

}  // namespace

extern "C" {

__attribute__((visibility("default"))) int bsa_diag_exp2(const float* x, float* y, int64_t n,
                                                         int32_t mode, void* stream) {
  if (x == nullptr || y == nullptr || n < 0 || (mode != 0 && mode != 1)) return -1;
  if (n == 0) return 0;
  const int64_t pairs = (n + 1) / 2;
  exp2_kernel<<<static_cast<unsigned>((pairs + 255) / 256), 256, 0,
                static_cast<cudaStream_t>(stream)>>>(x, y, n, mode);
  return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

// timeout_ns must lie in (0, 1 s]: the wait always runs to its limit.
__attribute__((visibility("default"))) int bsa_diag_unarmed_wait(int64_t timeout_ns,
                                                                 int32_t* err_word,
                                                                 long long* result,
                                                                 void* stream) {
  if (err_word == nullptr || result == nullptr) return -1;
  if (timeout_ns <= 0 || timeout_ns > 1000ll * 1000ll * 1000ll) return -1;
  unarmed_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<uint64_t>(timeout_ns), err_word, result);
  return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

}  // extern "C"
