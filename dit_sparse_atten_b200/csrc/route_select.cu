// (b) Route selection: persistence prior, top-mass rule, first-frame sink and
// the CSR pack, one CTA per (batch, head, query-block) row, writing the CSR
// route directly.
//
// Reference semantics:
//   prior      attention_backends/flex.py:535-541
//   top-mass   attention_backends/flex.py:83-94 (same rule sparse.py:171-181)
//   sink       attention_backends/flex.py:550-566
//   CSR pack   attention_backends/flex.py:275-281, layout_ops.py:55-83,128-151
//   keep       attention_backends/flex.py:473-493 (counter per group of rows)
//
// The kept set depends on the last bit of `sum(mass) * target` and of the
// prefix sums, so both follow the reference's PyTorch CPU evaluation order
// (ATen cascade sum with 8 float lanes and 4-way ILP; cumsum accumulated in
// float64 and rounded per prefix).  All float arithmetic on that path uses
// explicitly rounded intrinsics so nothing is contracted into an FMA.
// Equal values are ordered by ascending block id.
#include "route_common.cuh"

namespace bsa {
namespace {

__global__ void __launch_bounds__(kSelThreads) route_select_kernel(SelectArgs a, int np) {
  extern __shared__ __align__(16) uint8_t smem[];
  uint64_t* keys = reinterpret_cast<uint64_t*>(smem);                    // [np]
  float* vals = reinterpret_cast<float*>(keys + np);                     // [cols]
  uint8_t* flags = reinterpret_cast<uint8_t*>(vals + a.cols);            // [cols]
  __shared__ float s_threshold;
  __shared__ int s_count;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int64_t row = blockIdx.x;
  const int n = a.cols;
  const size_t base = static_cast<size_t>(row) * n;

  if (a.mass != nullptr) {
    for (int i = tid; i < n; i += kSelThreads) vals[i] = a.mass[base + i];
    __syncthreads();
    // ---- persistence prior: mass + p * mean(mass) * prev -------------------
    if (a.prev != nullptr && a.persistence != 0.f) {
      __shared__ float s_bump;
      if (warp == 0) {
        const float sum = torch_cpu_row_sum(vals, n);
        if (lane == 0) s_bump = __fmul_rn(a.persistence, __fdiv_rn(sum, static_cast<float>(n)));
      }
      __syncthreads();
      const float bump = s_bump;
      for (int i = tid; i < n; i += kSelThreads)
        vals[i] = __fadd_rn(vals[i], a.prev[base + i] ? bump : 0.f);
      __syncthreads();
    }
    // ---- threshold = sum * target ------------------------------------------
    if (warp == 0) {
      const float sum = torch_cpu_row_sum(vals, n);
      if (lane == 0) s_threshold = __fmul_rn(sum, a.target);
    }
    // ---- sort: value descending, block id ascending ------------------------
    sort_row_desc(vals, n, np, keys);
    // ---- count = #(cumsum < threshold) + 1, cumsum in float64 ---------------
    if (tid == 0) {
      const float thr = s_threshold;
      // Non-negative rows have monotone prefixes: stop at the first prefix
      // >= threshold or once the cap is reached.  Otherwise scan everything.
      const bool monotone = vals[key_id(keys[n - 1])] >= 0.f;
      double cs = 0.0;
      int below = 0;
      for (int r = 0; r < n; ++r) {
        cs = __dadd_rn(cs, static_cast<double>(vals[key_id(keys[r])]));
        if (__double2float_rn(cs) < thr) {
          ++below;
          if (monotone && below + 1 >= a.cap) break;
        } else if (monotone) {
          break;
        }
      }
      s_count = min(below + 1, a.cap);
    }
    __syncthreads();
    // Equal values straddling the cut: keep the ones the reference keeps.
    mark_first_desc(vals, n, s_count, keys, flags);
  } else {
    for (int i = tid; i < n; i += kSelThreads) flags[i] = a.route_in[base + i] ? 1 : 0;
    __syncthreads();
  }
  for (int i = tid; i < a.sink_blocks && i < n; i += kSelThreads) flags[i] = 1;
  __syncthreads();

  // ---- stable partition into CSR (selected ascending, then the rest) ------
  write_csr_row(flags, n, base, a.indices, a.route_out,
                a.counts != nullptr ? a.counts + row : nullptr,
                a.kept != nullptr ? a.kept + row / a.rows_per_group : nullptr);
}

}  // namespace

cudaError_t launch_route_select(const SelectArgs& a, cudaStream_t stream) {
  if (a.rows == 0) return cudaSuccess;
  if (a.cols <= 0 || a.cols > kMaxCols) return cudaErrorInvalidValue;
  int np = 1;
  while (np < a.cols) np <<= 1;
  const size_t smem = static_cast<size_t>(np) * 8 + static_cast<size_t>(a.cols) * 5 + 16;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(route_select_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  route_select_kernel<<<static_cast<unsigned>(a.rows), kSelThreads, smem, stream>>>(a, np);
  return cudaGetLastError();
}

}  // namespace bsa
