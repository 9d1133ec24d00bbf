// Row-selection helpers shared by the route-selection kernels (top-mass
// selection in route_select.cu, the directional budget update in
// directional.cu): the reference's PyTorch CPU float32 row sum, a block-wide
// sort of (value descending, block id ascending), the reference's unstable
// argsort tie order, and the CSR partition of a selected row; then the same
// steps for one warp per row (register bitonic sort of value keys).  Every
// block-wide function is called by all kSelThreads threads of the CTA, every
// warp_* function by all 32 lanes of a warp.
#pragma once

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

// The ordered sums below run on float (one sum) or float2 (two sums of the
// same length in one packed chain: each component is added exactly as a
// float sum would be).
__device__ __forceinline__ float sum_add(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float2 sum_add(float2 a, float2 b) { return __fadd2_rn(a, b); }
template <typename T>
__device__ __forceinline__ T sum_zero() {
  if constexpr (sizeof(T) == sizeof(float)) {
    return 0.f;
  } else {
    return make_float2(0.f, 0.f);
  }
}
__device__ __forceinline__ float sum_shfl(float v, int src) {
  return __shfl_sync(0xffffffffu, v, src);
}
__device__ __forceinline__ float2 sum_shfl(float2 v, int src) {
  return make_float2(__shfl_sync(0xffffffffu, v.x, src), __shfl_sync(0xffffffffu, v.y, src));
}

// Cascade over `size` items; item i of this lane is load(index(i)) (a float,
// or a float2 for two sums at once).  Items are loaded kBatch at a time ahead
// of their in-order additions.
template <int kBatch = 8, typename Load, typename IndexFn>
__device__ auto cascade_sum(Load load, int size, IndexFn index) {
  using T = decltype(load(0));
  static_assert(kBatch == 8 || kBatch == 16, "level_step is a multiple of 16");
  const int level_power = max(4, ceil_log2(size) / 4);
  const int level_step = 1 << level_power;
  const int level_mask = level_step - 1;
  T acc0 = sum_zero<T>(), acc1 = sum_zero<T>(), acc2 = sum_zero<T>(), acc3 = sum_zero<T>();
  int i = 0;
  while (i + level_step <= size) {
    // level_step is a power of two >= 16: items go in groups of kBatch, all
    // loaded before any is added (the additions keep their order).
    for (int j = 0; j < level_step; j += kBatch, i += kBatch) {
      T x[kBatch];
#pragma unroll
      for (int u = 0; u < kBatch; ++u) x[u] = load(index(i + u));
#pragma unroll
      for (int u = 0; u < kBatch; ++u) acc0 = sum_add(acc0, x[u]);
    }
    acc1 = sum_add(acc1, acc0);
    acc0 = sum_zero<T>();
    if ((i & (level_mask << level_power)) != 0) continue;
    acc2 = sum_add(acc2, acc1);
    acc1 = sum_zero<T>();
    if ((i & (level_mask << (2 * level_power))) != 0) continue;
    acc3 = sum_add(acc3, acc2);
    acc2 = sum_zero<T>();
  }
  for (; i < size; ++i) acc0 = sum_add(acc0, load(index(i)));
  acc0 = sum_add(acc0, acc1);
  acc0 = sum_add(acc0, acc2);
  acc0 = sum_add(acc0, acc3);
  return acc0;
}

// float32 sum of load(0..n-1) in the reference's CPU order (ATen's vectorised
// cascade: lane (k, v) of 4 accumulators x 8 float lanes takes items
// (4 i + k) * 8 + v, i.e. warp lane k * 8 + v takes items 32 i + lane);
// executed by one full warp, result valid in every lane.  A load returning
// float2 gives two such sums (of two rows of the same length) at once.
template <int kBatch = 8, typename Load>
__device__ auto torch_cpu_sum(Load load, int n) {
  using T = decltype(load(0));
  const int lane = threadIdx.x & 31;
  T result = sum_zero<T>();
  if (n < 8) {
    if (lane == 0) {
      const int size_ilp = n / 4;
      T p[4];
#pragma unroll
      for (int k = 0; k < 4; ++k)
        p[k] = cascade_sum(load, size_ilp, [k](int i) { return 4 * i + k; });
      for (int i = size_ilp * 4; i < n; ++i) p[0] = sum_add(p[0], load(i));
#pragma unroll
      for (int k = 1; k < 4; ++k) p[0] = sum_add(p[0], p[k]);
      result = sum_add(sum_zero<T>(), p[0]);
    }
    return sum_shfl(result, 0);
  }
  const int vec_size = n / 8;
  const int size_ilp = vec_size / 4;
  const int k = lane >> 3;
  const int v = lane & 7;
  T acc = cascade_sum<kBatch>(load, size_ilp, [k, v](int i) { return (4 * i + k) * 8 + v; });
  if (k == 0)
    for (int i = size_ilp * 4; i < vec_size; ++i) acc = sum_add(acc, load(i * 8 + v));
  const T a1 = sum_shfl(acc, (v + 8) & 31);
  const T a2 = sum_shfl(acc, (v + 16) & 31);
  const T a3 = sum_shfl(acc, (v + 24) & 31);
  T p = sum_add(sum_add(sum_add(acc, a1), a2), a3);
  T f = sum_zero<T>();
  if (lane == 0)
    for (int i = vec_size * 8; i < n; ++i) f = sum_add(f, load(i));
  for (int l = 0; l < 8; ++l) {
    const T pl = sum_shfl(p, l);
    if (lane == 0) f = sum_add(f, pl);
  }
  return sum_shfl(f, 0);
}

// float32 row sum of x[0..n-1] in the reference's CPU order (one full warp).
__device__ float torch_cpu_row_sum(const float* x, int n) {
  return torch_cpu_sum([x](int i) { return x[i]; }, n);
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

// Sort key: value descending, then block id ascending.
__device__ __forceinline__ uint64_t desc_key(float v, int i) {
  return (static_cast<uint64_t>(~float_order_key(v)) << 32) | static_cast<uint32_t>(i);
}

__device__ __forceinline__ int key_id(uint64_t key) { return static_cast<int>(key & 0xffffffffu); }

// keys[0, np) <- sorted desc_key(vals[i], i) for i < n, padding (~0) after;
// np is the power of two >= n.
__device__ void sort_row_desc(const float* vals, int n, int np, uint64_t* keys) {
  const int tid = threadIdx.x;
  for (int i = tid; i < np; i += kSelThreads) keys[i] = i < n ? desc_key(vals[i], i) : ~0ull;
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
}

// flags[i] = 1 for the first `count` entries of the reference's
// `vals.argsort(descending=True)`, 0 for the rest.  keys holds the output of
// sort_row_desc(vals); where equal values straddle the cut one thread replays
// the reference's introsort (keys is reused as its scratch).
__device__ void mark_first_desc(const float* vals, int n, int count, uint64_t* keys,
                                uint8_t* flags) {
  const int tid = threadIdx.x;
  const bool tie = count > 0 && count < n &&
                   vals[key_id(keys[count - 1])] == vals[key_id(keys[count])];
  if (!tie) {
    for (int r = tid; r < n; r += kSelThreads) flags[key_id(keys[r])] = r < count ? 1 : 0;
  } else {
    SortPair* pairs = reinterpret_cast<SortPair*>(keys);
    __syncthreads();
    if (tid == 0) {
      for (int i = 0; i < n; ++i) pairs[i] = SortPair{vals[i], i};
      introsort_desc(pairs, n);
    }
    __syncthreads();
    for (int r = tid; r < n; r += kSelThreads) flags[pairs[r].i] = r < count ? 1 : 0;
  }
  __syncthreads();
}

// Stable partition of a row's flags into CSR (selected ids ascending, then
// the rest); writes any of indices / route_out (at row offset base), the count
// and the kept counter that are non-null.
__device__ void write_csr_row(const uint8_t* flags, int n, size_t base, int32_t* indices,
                              uint8_t* route_out, int32_t* count_out,
                              unsigned long long* kept_slot) {
  __shared__ int s_warp_tot[kSelThreads / 32];
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
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
    if (indices != nullptr) {
      const int pos = f ? sel_before : total + (i - sel_before);
      indices[base + pos] = i;
    }
    if (route_out != nullptr) route_out[base + i] = static_cast<uint8_t>(f);
    sel_before += f;
  }
  if (tid == 0) {
    if (count_out != nullptr) *count_out = total;
    if (kept_slot != nullptr) atomicAdd(kept_slot, static_cast<unsigned long long>(total));
  }
}


// ---------------------------------------------------------------------------
// Warp-per-row helpers (rows of up to kWarpSelMaxCols blocks).  A row's values
// sit in shared memory at vidx(e) (one pad word per 16, so lane-major register
// loads are conflict-free); sort keys live in registers, ITEMS per lane, lane l
// holding positions [l*ITEMS, (l+1)*ITEMS).  Called by all 32 lanes.
// ---------------------------------------------------------------------------
constexpr int kWarpSelMaxCols = 512;
constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ int vidx(int e) { return e + (e >> 4); }

// Ascending in this key = descending in value (-0 and +0 share a key).
__device__ __forceinline__ uint32_t desc_value_key(float v) { return ~float_order_key(v); }

__device__ __forceinline__ float desc_key_value(uint32_t key) {
  const uint32_t k = ~key;
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

template <int ITEMS>
__device__ __forceinline__ void warp_sort_ascending(uint32_t (&k)[ITEMS]) {
  const int lane = threadIdx.x & 31;
  constexpr int kLog = (ITEMS == 1 ? 5 : ITEMS == 2 ? 6 : ITEMS == 4 ? 7 : ITEMS == 8 ? 8 : 9);
#pragma unroll
  for (int ls = 1; ls <= kLog; ++ls) {
    const int size = 1 << ls;
    uint32_t flip[ITEMS];
#pragma unroll
    for (int j = 0; j < ITEMS; ++j) {
      flip[j] = ((lane * ITEMS + j) & size) ? 0xffffffffu : 0u;   // 0 in the last phase
      k[j] ^= flip[j];
    }
#pragma unroll
    for (int ss = ls - 1; ss >= 0; --ss) {
      const int stride = 1 << ss;
      if (stride < ITEMS) {
#pragma unroll
        for (int j = 0; j < ITEMS; ++j) {
          if (j & stride) continue;
          const uint32_t x = k[j], y = k[j | stride];
          k[j] = min(x, y);
          k[j | stride] = max(x, y);
        }
      } else {
        const int lstride = stride / ITEMS;
        const bool lower = (lane & lstride) == 0;
#pragma unroll
        for (int j = 0; j < ITEMS; ++j) {
          const uint32_t o = __shfl_xor_sync(kFull, k[j], lstride);
          k[j] = lower ? min(k[j], o) : max(k[j], o);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < ITEMS; ++j) k[j] ^= flip[j];
  }
}

// Element pos (0 <= pos < 32*ITEMS) of a per-lane register array.
template <int ITEMS, typename T>
__device__ __forceinline__ T lane_item(const T (&x)[ITEMS], int pos) {
  const int lane = threadIdx.x & 31;
  T v = T(0);
#pragma unroll
  for (int j = 0; j < ITEMS; ++j)
    if (lane * ITEMS + j == pos) v = x[j];
  return __shfl_sync(kFull, v, pos / ITEMS);
}


// Bitonic network of 32*ITEMS keys for one warp.
template <int ITEMS>
__device__ __forceinline__ void warp_load_sorted_keys(const float* vals, int n,
                                                      uint32_t (&key)[ITEMS]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < ITEMS; ++j) {
    const int e = lane * ITEMS + j;
    key[j] = e < n ? desc_value_key(vals[vidx(e)]) : 0xffffffffu;
  }
  warp_sort_ascending<ITEMS>(key);
}

// flags[i] = 1 for the first `count` entries of the reference's
// `vals.argsort(descending=True)` (vals at vidx(i)), 0 for the rest, given the
// sort key `cut` of the value at position count - 1 and whether equal values
// straddle the cut (then lane 0 replays the reference's introsort in `pairs`).
__device__ void warp_flags_from_cut(const float* vals, int n, int count, uint32_t cut, bool tie,
                                    SortPair* pairs, uint8_t* flags) {
  const int lane = threadIdx.x & 31;
  if (!tie) {
    for (int i = lane; i < n; i += 32) flags[i] = desc_value_key(vals[vidx(i)]) <= cut ? 1 : 0;
  } else {
    __syncwarp();
    if (lane == 0) {
      for (int i = 0; i < n; ++i) pairs[i] = SortPair{vals[vidx(i)], i};
      introsort_desc(pairs, n);
    }
    __syncwarp();
    for (int r = lane; r < n; r += 32) flags[pairs[r].i] = r < count ? 1 : 0;
  }
  __syncwarp();
}

// Warp version of mark_first_desc: sorts the row itself.
template <int ITEMS>
__device__ void warp_mark_first_desc(const float* vals, int n, int count, SortPair* pairs,
                                     uint8_t* flags) {
  const int lane = threadIdx.x & 31;
  if (count >= n || count <= 0) {
    for (int i = lane; i < n; i += 32) flags[i] = count > 0 ? 1 : 0;
    __syncwarp();
    return;
  }
  uint32_t key[ITEMS];
  warp_load_sorted_keys<ITEMS>(vals, n, key);
  const uint32_t cut = lane_item<ITEMS>(key, count - 1);
  const bool tie = lane_item<ITEMS>(key, count) == cut;
  warp_flags_from_cut(vals, n, count, cut, tie, pairs, flags);
}

// Warp version of write_csr_row (same outputs).
__device__ void warp_write_csr_row(const uint8_t* flags, int n, size_t base, int32_t* indices,
                                   uint8_t* route_out, int32_t* count_out,
                                   unsigned long long* kept_slot) {
  const int lane = threadIdx.x & 31;
  int total = 0;
  for (int i0 = 0; i0 < n; i0 += 32) {
    const int i = i0 + lane;
    total += __popc(__ballot_sync(kFull, i < n && flags[i] != 0));
  }
  const unsigned below_mask = (1u << lane) - 1u;
  int sel = 0;
  for (int i0 = 0; i0 < n; i0 += 32) {
    const int i = i0 + lane;
    const bool f = i < n && flags[i] != 0;
    const unsigned m = __ballot_sync(kFull, f);
    const int before = sel + __popc(m & below_mask);
    if (i < n) {
      if (indices != nullptr) indices[base + (f ? before : total + (i - before))] = i;
      if (route_out != nullptr) route_out[base + i] = static_cast<uint8_t>(f);
    }
    sel += __popc(m);
  }
  if (lane == 0) {
    if (count_out != nullptr) *count_out = total;
    if (kept_slot != nullptr) atomicAdd(kept_slot, static_cast<unsigned long long>(total));
  }
}

}  // namespace
}  // namespace bsa
