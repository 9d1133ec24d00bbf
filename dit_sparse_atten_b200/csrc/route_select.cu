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
#include "bsa_kernels.h"

namespace bsa {
namespace {

constexpr int kSelThreads = 128;
constexpr int kMaxCols = 4096;

__device__ __forceinline__ uint32_t float_order_key(float v) {
  if (v == 0.0f) v = 0.0f;  // -0 and +0 compare equal: one key
  const uint32_t u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ int ceil_log2(int v) {
  return v <= 1 ? 0 : 32 - __clz(v - 1);
}

// Cascade over `size` items; item i of this lane is x[index(i)].
template <typename IndexFn>
__device__ float cascade_sum(const float* x, int size, IndexFn index) {
  const int level_power = max(4, ceil_log2(size) / 4);
  const int level_step = 1 << level_power;
  const int level_mask = level_step - 1;
  float acc0 = 0.f, acc1 = 0.f, acc2 = 0.f, acc3 = 0.f;
  int i = 0;
  while (i + level_step <= size) {
    for (int j = 0; j < level_step; ++j, ++i) acc0 = __fadd_rn(acc0, x[index(i)]);
    acc1 = __fadd_rn(acc1, acc0);
    acc0 = 0.f;
    if ((i & (level_mask << level_power)) != 0) continue;
    acc2 = __fadd_rn(acc2, acc1);
    acc1 = 0.f;
    if ((i & (level_mask << (2 * level_power))) != 0) continue;
    acc3 = __fadd_rn(acc3, acc2);
    acc2 = 0.f;
  }
  for (; i < size; ++i) acc0 = __fadd_rn(acc0, x[index(i)]);
  acc0 = __fadd_rn(acc0, acc1);
  acc0 = __fadd_rn(acc0, acc2);
  acc0 = __fadd_rn(acc0, acc3);
  return acc0;
}

// float32 row sum in the reference's CPU order; executed by one full warp,
// result valid in every lane.
__device__ float torch_cpu_row_sum(const float* x, int n) {
  const int lane = threadIdx.x & 31;
  float result = 0.f;
  if (n < 8) {
    if (lane == 0) {
      const int size_ilp = n / 4;
      float p[4];
      for (int k = 0; k < 4; ++k)
        p[k] = cascade_sum(x, size_ilp, [k](int i) { return 4 * i + k; });
      for (int i = size_ilp * 4; i < n; ++i) p[0] = __fadd_rn(p[0], x[i]);
      for (int k = 1; k < 4; ++k) p[0] = __fadd_rn(p[0], p[k]);
      result = __fadd_rn(0.f, p[0]);
    }
    return __shfl_sync(0xffffffffu, result, 0);
  }
  const int vec_size = n / 8;
  const int size_ilp = vec_size / 4;
  const int k = lane >> 3;
  const int v = lane & 7;
  float acc = cascade_sum(x, size_ilp, [k, v](int i) { return (4 * i + k) * 8 + v; });
  if (k == 0)
    for (int i = size_ilp * 4; i < vec_size; ++i) acc = __fadd_rn(acc, x[i * 8 + v]);
  const float a1 = __shfl_sync(0xffffffffu, acc, (v + 8) & 31);
  const float a2 = __shfl_sync(0xffffffffu, acc, (v + 16) & 31);
  const float a3 = __shfl_sync(0xffffffffu, acc, (v + 24) & 31);
  float p = __fadd_rn(__fadd_rn(__fadd_rn(acc, a1), a2), a3);
  float f = 0.f;
  if (lane == 0)
    for (int i = vec_size * 8; i < n; ++i) f = __fadd_rn(f, x[i]);
  for (int l = 0; l < 8; ++l) {
    const float pl = __shfl_sync(0xffffffffu, p, l);
    if (lane == 0) f = __fadd_rn(f, pl);
  }
  return __shfl_sync(0xffffffffu, f, 0);
}

// ---------------------------------------------------------------------------
// Tie order of the reference's unstable `argsort(descending=True)`.
// The reference sorts (value, index) pairs with libstdc++'s introsort and a
// key-only greater-than comparator, so equal values end up in the order that
// algorithm leaves them.  The count of kept blocks does not depend on it (the
// sorted value sequence is the same), only which of several equal values
// straddling the cut are kept; for those rows one thread replays the
// introsort.  Published algorithm: median-of-three quicksort with unguarded
// partitions, heapsort below a depth limit of 2*floor(log2 n), then insertion
// sort with a 16-element threshold.
// ---------------------------------------------------------------------------
struct SortPair {
  float v;
  int32_t i;
};

__device__ __forceinline__ bool pair_greater(const SortPair& x, const SortPair& y) {
  return x.v > y.v;
}

__device__ __forceinline__ void pair_swap(SortPair* a, int x, int y) {
  const SortPair t = a[x];
  a[x] = a[y];
  a[y] = t;
}

__device__ void move_median_to_first(SortPair* a, int result, int x, int y, int z) {
  if (pair_greater(a[x], a[y])) {
    if (pair_greater(a[y], a[z])) pair_swap(a, result, y);
    else if (pair_greater(a[x], a[z])) pair_swap(a, result, z);
    else pair_swap(a, result, x);
  } else if (pair_greater(a[x], a[z])) {
    pair_swap(a, result, x);
  } else if (pair_greater(a[y], a[z])) {
    pair_swap(a, result, z);
  } else {
    pair_swap(a, result, y);
  }
}

__device__ int unguarded_partition(SortPair* a, int first, int last, int pivot) {
  for (;;) {
    while (pair_greater(a[first], a[pivot])) ++first;
    --last;
    while (pair_greater(a[pivot], a[last])) --last;
    if (!(first < last)) return first;
    pair_swap(a, first, last);
    ++first;
  }
}

__device__ void adjust_heap(SortPair* a, int first, int hole, int len, SortPair value) {
  const int top = hole;
  int second = hole;
  while (second < (len - 1) / 2) {
    second = 2 * (second + 1);
    if (pair_greater(a[first + second], a[first + second - 1])) --second;
    a[first + hole] = a[first + second];
    hole = second;
  }
  if ((len & 1) == 0 && second == (len - 2) / 2) {
    second = 2 * (second + 1);
    a[first + hole] = a[first + second - 1];
    hole = second - 1;
  }
  int parent = (hole - 1) / 2;
  while (hole > top && pair_greater(a[first + parent], value)) {
    a[first + hole] = a[first + parent];
    hole = parent;
    parent = (hole - 1) / 2;
  }
  a[first + hole] = value;
}

__device__ void heap_sort(SortPair* a, int first, int last) {
  const int len = last - first;
  if (len >= 2) {
    for (int parent = (len - 2) / 2;; --parent) {
      adjust_heap(a, first, parent, len, a[first + parent]);
      if (parent == 0) break;
    }
  }
  while (last - first > 1) {
    --last;
    const SortPair value = a[last];
    a[last] = a[first];
    adjust_heap(a, first, 0, last - first, value);
  }
}

__device__ void unguarded_linear_insert(SortPair* a, int last) {
  const SortPair val = a[last];
  int next = last - 1;
  while (pair_greater(val, a[next])) {
    a[last] = a[next];
    last = next;
    --next;
  }
  a[last] = val;
}

__device__ void introsort_desc(SortPair* a, int n) {
  constexpr int kThreshold = 16;
  if (n <= 0) return;
  int st_first[64], st_last[64], st_depth[64];
  int sp = 0;
  st_first[0] = 0;
  st_last[0] = n;
  st_depth[0] = 2 * (31 - __clz(n));
  sp = 1;
  // Disjoint subranges are independent, so a stack replaces the recursion.
  while (sp > 0) {
    --sp;
    const int first = st_first[sp];
    int last = st_last[sp];
    int depth = st_depth[sp];
    while (last - first > kThreshold) {
      if (depth == 0) {
        heap_sort(a, first, last);
        break;
      }
      --depth;
      const int mid = first + (last - first) / 2;
      move_median_to_first(a, first, first + 1, mid, last - 1);
      const int cut = unguarded_partition(a, first + 1, last, first);
      st_first[sp] = cut;
      st_last[sp] = last;
      st_depth[sp] = depth;
      ++sp;
      last = cut;
    }
  }
  const int head = n > kThreshold ? kThreshold : n;
  for (int i = 1; i < head; ++i) {
    if (pair_greater(a[i], a[0])) {
      const SortPair val = a[i];
      for (int j = i; j > 0; --j) a[j] = a[j - 1];
      a[0] = val;
    } else {
      unguarded_linear_insert(a, i);
    }
  }
  for (int i = head; i < n; ++i) unguarded_linear_insert(a, i);
}

__global__ void __launch_bounds__(kSelThreads) route_select_kernel(SelectArgs a, int np) {
  extern __shared__ __align__(16) uint8_t smem[];
  uint64_t* keys = reinterpret_cast<uint64_t*>(smem);                    // [np]
  float* vals = reinterpret_cast<float*>(keys + np);                     // [cols]
  uint8_t* flags = reinterpret_cast<uint8_t*>(vals + a.cols);            // [cols]
  __shared__ float s_threshold;
  __shared__ int s_count;
  __shared__ bool s_tie;
  __shared__ int s_warp_tot[kSelThreads / 32];

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
    for (int i = tid; i < np; i += kSelThreads)
      keys[i] = i < n ? ((static_cast<uint64_t>(~float_order_key(vals[i])) << 32) |
                         static_cast<uint32_t>(i))
                      : ~0ull;
    __syncthreads();
    for (int size = 2; size <= np; size <<= 1) {
      for (int stride = size >> 1; stride > 0; stride >>= 1) {
        for (int p = tid; p < (np >> 1); p += kSelThreads) {
          const int lo = ((p / stride) * stride << 1) + (p % stride);
          const int hi = lo + stride;
          const bool ascending = (lo & size) == 0;
          const uint64_t x = keys[lo], y = keys[hi];
          if ((x > y) == ascending) {
            keys[lo] = y;
            keys[hi] = x;
          }
        }
        __syncthreads();
      }
    }
    // ---- count = #(cumsum < threshold) + 1, cumsum in float64 ---------------
    if (tid == 0) {
      const float thr = s_threshold;
      // Non-negative rows have monotone prefixes: stop at the first prefix
      // >= threshold or once the cap is reached.  Otherwise scan everything.
      const bool monotone = vals[static_cast<int>(keys[n - 1] & 0xffffffffu)] >= 0.f;
      double cs = 0.0;
      int below = 0;
      for (int r = 0; r < n; ++r) {
        cs = __dadd_rn(cs, static_cast<double>(vals[static_cast<int>(keys[r] & 0xffffffffu)]));
        if (__double2float_rn(cs) < thr) {
          ++below;
          if (monotone && below + 1 >= a.cap) break;
        } else if (monotone) {
          break;
        }
      }
      const int count = min(below + 1, a.cap);
      s_count = count;
      s_tie = count < n && vals[static_cast<int>(keys[count - 1] & 0xffffffffu)] ==
                               vals[static_cast<int>(keys[count] & 0xffffffffu)];
    }
    __syncthreads();
    const int count = s_count;
    if (!s_tie) {
      for (int r = tid; r < n; r += kSelThreads)
        flags[static_cast<int>(keys[r] & 0xffffffffu)] = r < count ? 1 : 0;
    } else {
      // Equal values straddle the cut: keep the ones the reference keeps.
      SortPair* pairs = reinterpret_cast<SortPair*>(keys);
      if (tid == 0) {
        for (int i = 0; i < n; ++i) pairs[i] = SortPair{vals[i], i};
        introsort_desc(pairs, n);
      }
      __syncthreads();
      for (int r = tid; r < n; r += kSelThreads) flags[pairs[r].i] = r < count ? 1 : 0;
    }
    __syncthreads();
  } else {
    for (int i = tid; i < n; i += kSelThreads) flags[i] = a.route_in[base + i] ? 1 : 0;
    __syncthreads();
  }
  for (int i = tid; i < a.sink_blocks && i < n; i += kSelThreads) flags[i] = 1;
  __syncthreads();

  // ---- stable partition into CSR (selected ascending, then the rest) ------
  const int per = (n + kSelThreads - 1) / kSelThreads;
  const int begin = min(n, tid * per);
  const int end = min(n, begin + per);
  int local = 0;
  for (int i = begin; i < end; ++i) local += flags[i];
  int incl = local;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += y;
  }
  if (lane == 31) s_warp_tot[warp] = incl;
  __syncthreads();
  int warp_off = 0, total = 0;
  for (int w = 0; w < kSelThreads / 32; ++w) {
    if (w < warp) warp_off += s_warp_tot[w];
    total += s_warp_tot[w];
  }
  int sel_before = warp_off + incl - local;
  for (int i = begin; i < end; ++i) {
    const int f = flags[i];
    if (a.indices != nullptr) {
      const int pos = f ? sel_before : total + (i - sel_before);
      a.indices[base + pos] = i;
    }
    if (a.route_out != nullptr) a.route_out[base + i] = static_cast<uint8_t>(f);
    sel_before += f;
  }
  if (tid == 0) {
    if (a.counts != nullptr) a.counts[row] = total;
    if (a.kept != nullptr)
      atomicAdd(a.kept + row / a.rows_per_group, static_cast<unsigned long long>(total));
  }
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
