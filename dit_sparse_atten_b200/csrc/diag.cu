// Element-wise evaluation of the two exp2 paths the softmax kernels use, so
// tests can check their accuracy directly (bsa_exp2 in include/bsa.h).
#include "bsa_kernels.h"

namespace bsa {
namespace {

__global__ void exp2_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t n,
                            int mode) {
  const int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 2;
  if (i >= n) return;
  const float x0 = x[i];
  const float x1 = i + 1 < n ? x[i + 1] : 0.f;
  float2 r;
  if (mode == 1) {
    r = exp2_poly2(make_float2(x0, x1));
  } else {
    r = make_float2(ex2_approx(x0), ex2_approx(x1));
  }
  y[i] = r.x;
  if (i + 1 < n) y[i + 1] = r.y;
}

}  // namespace

cudaError_t launch_exp2(const float* x, float* y, int64_t n, int mode, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  const int64_t pairs = (n + 1) / 2;
  exp2_kernel<<<static_cast<unsigned>((pairs + 255) / 256), 256, 0, stream>>>(x, y, n, mode);
  return cudaGetLastError();
}

}  // namespace bsa
