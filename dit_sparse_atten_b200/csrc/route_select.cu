// (b) Route selection: persistence prior, top-mass rule, first-frame sink and
// the CSR pack per (batch, head, query-block) row, writing the CSR route
// directly: one warp per row up to 512 blocks (route_select_warp_kernel),
// one CTA per row above that (route_select_kernel).
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
// The CTA kernel's sort orders equal values by ascending block id.
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

// ---------------------------------------------------------------------------
// Warp-per-row selection for rows of up to 512 blocks (every Wan layout).
//
// One warp owns a row and needs no block barrier.  The sort is a register
// bitonic network over 32-bit order keys of the values alone, ITEMS per lane
// (lane l holds sorted positions [l*ITEMS, (l+1)*ITEMS)); each merge phase
// complements the keys of its descending halves so that every exchange is an
// ascending min/max pair.  Block ids do not travel with the keys: once the
// count is known, the kept set is every block whose value is at least the
// value at the cut -- unless equal values straddle the cut, where the
// reference's introsort order decides and lane 0 replays it.
//
// The count rule needs the reference's float64 prefix sums taken in sorted
// order.  For a non-negative row those are exact -- and therefore equal to
// any parallel evaluation -- as long as every prefix up to the cut is a sum
// of floats that are multiples of the ulp of the smallest of them and stays
// below 2^53 of those ulps.  The warp checks that condition (with a factor-2
// margin) at the last prefix the rule looks at; rows that fail it, rows with
// negative values and rows with NaN/inf take the serial scan of lane 0 over
// the same sorted values, as the CTA kernel does.
// ---------------------------------------------------------------------------
constexpr int kWarpSelWarps = 4;            // rows per CTA

struct WarpSelSmem {
  union {
    uint32_t keys[kWarpSelMaxCols];          // sorted keys for the serial scan
    SortPair pairs[kWarpSelMaxCols];         // tie replay
  };
  float vals[kWarpSelMaxCols + kWarpSelMaxCols / 16];   // element e at vidx(e)
  uint8_t flags[kWarpSelMaxCols];
};

template <int ITEMS>
__global__ void __launch_bounds__(kWarpSelWarps * 32, 8) route_select_warp_kernel(SelectArgs a) {
  __shared__ WarpSelSmem smem_all[kWarpSelWarps];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kWarpSelWarps + warp;
  if (row >= a.rows) return;  // warp-uniform; the kernel has no CTA barrier
  WarpSelSmem& sm = smem_all[warp];
  float* vals = sm.vals;
  uint8_t* flags = sm.flags;
  const int n = a.cols;
  const size_t base = static_cast<size_t>(row) * n;
  const auto load = [vals](int i) { return vals[vidx(i)]; };

  if (a.mass != nullptr) {
    for (int i = lane; i < n; i += 32) vals[vidx(i)] = a.mass[base + i];
    __syncwarp();
    // ---- persistence prior: mass + p * mean(mass) * prev -------------------
    if (a.prev != nullptr && a.persistence != 0.f) {
      const float sum = torch_cpu_sum(load, n);
      const float bump = __fmul_rn(a.persistence, __fdiv_rn(sum, static_cast<float>(n)));
      __syncwarp();
      for (int i = lane; i < n; i += 32)
        vals[vidx(i)] = __fadd_rn(vals[vidx(i)], a.prev[base + i] ? bump : 0.f);
      __syncwarp();
    }
    const float thr = __fmul_rn(torch_cpu_sum(load, n), a.target);

    // ---- sort the values descending ------------------------------------------
    uint32_t key[ITEMS];
    warp_load_sorted_keys<ITEMS>(vals, n, key);
    float v[ITEMS];
#pragma unroll
    for (int j = 0; j < ITEMS; ++j) v[j] = lane * ITEMS + j < n ? desc_key_value(key[j]) : 0.f;

    // ---- prefix sums (float64) and the first prefix >= threshold -------------
    double lane_sum = 0.0;
#pragma unroll
    for (int j = 0; j < ITEMS; ++j) lane_sum = __dadd_rn(lane_sum, static_cast<double>(v[j]));
    double incl = lane_sum;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const double y = __shfl_up_sync(kFull, incl, off);
      if (lane >= off) incl = __dadd_rn(incl, y);
    }
    double excl = __shfl_up_sync(kFull, incl, 1);
    if (lane == 0) excl = 0.0;
    const bool monotone = lane_item<ITEMS>(v, n - 1) >= 0.f;
    int first = n;
    {
      double cs = excl;
#pragma unroll
      for (int j = 0; j < ITEMS; ++j) {
        cs = __dadd_rn(cs, static_cast<double>(v[j]));
        if (first == n && lane * ITEMS + j < n && !(__double2float_rn(cs) < thr))
          first = lane * ITEMS + j;
      }
    }
    const int c = __reduce_min_sync(kFull, first);
    bool fast = monotone;
    int count = min(c + 1, a.cap);
    // Last prefix the serial rule evaluates: the crossing, or cap - 2 where
    // the cap stops it first (cap == 1 keeps one block whatever the sums).
    const int check = a.cap >= 2 ? min(c, a.cap - 2) : -1;
    if (fast && check >= 0) {
      const float x = lane_item<ITEMS>(v, check);
      double cs = excl, s_lane = 0.0;
#pragma unroll
      for (int j = 0; j < ITEMS; ++j) {
        cs = __dadd_rn(cs, static_cast<double>(v[j]));
        if (lane * ITEMS + j == check) s_lane = cs;
      }
      const double s = __shfl_sync(kFull, s_lane, check / ITEMS);
      if (!(x > 0.f && x <= 3.402823466e38f)) {
        fast = false;
      } else {
        // ulp(x) = 2^(max(e, 1) - 150); exact while s <= 2^52 ulp(x)
        const int e = static_cast<int>((__float_as_uint(x) >> 23) & 0xffu);
        const double limit =
            __longlong_as_double(static_cast<long long>(max(e, 1) - 98 + 1023) << 52);
        if (!(s <= limit)) fast = false;
      }
    }
    if (!fast) {
#pragma unroll
      for (int j = 0; j < ITEMS; ++j) sm.keys[lane * ITEMS + j] = desc_value_key(v[j]);
      __syncwarp();
      int cnt = 0;
      if (lane == 0) {
        double cs = 0.0;
        int below = 0;
        for (int r = 0; r < n; ++r) {
          cs = __dadd_rn(cs, static_cast<double>(desc_key_value(sm.keys[r])));
          if (__double2float_rn(cs) < thr) {
            ++below;
            if (monotone && below + 1 >= a.cap) break;
          } else if (monotone) {
            break;
          }
        }
        cnt = min(below + 1, a.cap);
      }
      count = __shfl_sync(kFull, cnt, 0);
      __syncwarp();
    }

    // ---- kept set -------------------------------------------------------------
    const uint32_t cut = desc_value_key(lane_item<ITEMS>(v, count - 1));
    const bool tie = count < n && desc_value_key(lane_item<ITEMS>(v, count)) == cut;
    warp_flags_from_cut(vals, n, count, cut, tie, sm.pairs, flags);
  } else {
    for (int i = lane; i < n; i += 32) flags[i] = a.route_in[base + i] ? 1 : 0;
  }
  __syncwarp();
  for (int i = lane; i < a.sink_blocks && i < n; i += 32) flags[i] = 1;
  __syncwarp();

  warp_write_csr_row(flags, n, base, a.indices, a.route_out,
                     a.counts != nullptr ? a.counts + row : nullptr,
                     a.kept != nullptr ? a.kept + row / a.rows_per_group : nullptr);
}

template <int ITEMS>
cudaError_t launch_warp_select(const SelectArgs& a, cudaStream_t stream) {
  const int64_t ctas = (a.rows + kWarpSelWarps - 1) / kWarpSelWarps;
  route_select_warp_kernel<ITEMS>
      <<<static_cast<unsigned>(ctas), kWarpSelWarps * 32, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_route_select(const SelectArgs& a, cudaStream_t stream) {
  if (a.rows == 0) return cudaSuccess;
  if (a.cols <= 0 || a.cols > kMaxCols) return cudaErrorInvalidValue;
  if (a.cols <= 32) return launch_warp_select<1>(a, stream);
  if (a.cols <= 64) return launch_warp_select<2>(a, stream);
  if (a.cols <= 128) return launch_warp_select<4>(a, stream);
  if (a.cols <= 256) return launch_warp_select<8>(a, stream);
  if (a.cols <= kWarpSelMaxCols) return launch_warp_select<16>(a, stream);
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
