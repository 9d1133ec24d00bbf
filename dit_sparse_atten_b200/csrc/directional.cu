// (f3) Directional frontier update of a route: expand the previous route's
// frontier by one best unselected spatial neighbour per cell, optionally add
// the highest-mass cells outside the pool, then keep a per-row budget of the
// highest prior scores inside the pool; first-frame sink; CSR; frontier of the
// new route.  A plane is one (batch, head) route [n, n]; neighbours [n, 4] are
// shared by the query and the key axis (the route is square).
//
// Reference semantics (attention_backends/):
//   frontier        routing.py:10-43
//   best targets    routing.py:55-84   (first of equal maxima, Tensor.max)
//   budget select   routing.py:87-94
//   update          routing.py:97-168
//   caller / sink   flex.py:517-534, flex.py:550-566
//
// Three launches on the caller's stream:
//   1. candidate_scatter_kernel, one thread per cell: for each frontier cell
//      the best neighbour along Q and along K, eligibility, and the scatter of
//      the Q, K and joint candidates (byte stores of 1; concurrent stores to a
//      cell write the same value).
//   2. directional_select_warp_kernel (one warp per row, n <= 512) or
//      directional_select_kernel (one CTA per row): candidates & ~prev, pool,
//      exploration, prior score, fixed budget, sink, CSR, kept counter.
//   3. frontier_kernel over the new route (only when a frontier is wanted).
// Float arithmetic whose last bit decides a route follows the reference's
// PyTorch CPU evaluation order (route_common.cuh) with explicitly rounded
// intrinsics.
#include "route_common.cuh"

namespace bsa {
namespace {

constexpr int kCellThreads = 256;

// Ids outside [-1, n) are reported and treated as "no neighbour".
__device__ __forceinline__ int checked_block(int t, int n, int* err_word) {
  if (t < -1 || t >= n) {
    if (err_word) atomicOr(err_word, kErrBadRoute);
    return -1;
  }
  return t;
}

__device__ __forceinline__ int4 load_neighbors(const int32_t* nb, int block, int n,
                                               int* err_word) {
  const int4 t = __ldg(reinterpret_cast<const int4*>(nb) + block);
  return make_int4(checked_block(t.x, n, err_word), checked_block(t.y, n, err_word),
                   checked_block(t.z, n, err_word), checked_block(t.w, n, err_word));
}

__device__ __forceinline__ int nb_at(const int4& t, int d) {
  return d == 0 ? t.x : d == 1 ? t.y : d == 2 ? t.z : t.w;
}

// Cell (q, k) of a plane is on the frontier: selected, with a valid neighbour
// along Q (row t, same column) or along K (same row, column t) unselected.
__device__ __forceinline__ bool on_frontier(const uint8_t* plane, int n, int q, int k,
                                            const int4& nq, const int4& nk) {
  if (!plane[static_cast<size_t>(q) * n + k]) return false;
#pragma unroll
  for (int d = 0; d < 4; ++d) {
    const int t = nb_at(nq, d);
    if (t >= 0 && !plane[static_cast<size_t>(t) * n + k]) return true;
  }
#pragma unroll
  for (int d = 0; d < 4; ++d) {
    const int t = nb_at(nk, d);
    if (t >= 0 && !plane[static_cast<size_t>(q) * n + t]) return true;
  }
  return false;
}

__global__ void __launch_bounds__(kCellThreads) frontier_kernel(const uint8_t* __restrict__ route,
                                                                const int32_t* __restrict__ nb,
                                                                int64_t planes, int n,
                                                                uint8_t* __restrict__ out,
                                                                int* err_word) {
  // One CTA per (plane, q) row at a time, threads across k: the row's
  // coordinates and Q neighbours are computed once per row, not per cell.
  const int64_t rows = planes * n;
  for (int64_t pq = blockIdx.x; pq < rows; pq += gridDim.x) {
    const int q = static_cast<int>(pq % n);
    const uint8_t* plane = route + (pq - q) * n;
    const int4 nq = load_neighbors(nb, q, n, err_word);
    for (int k = threadIdx.x; k < n; k += kCellThreads) {
      const int4 nk = load_neighbors(nb, k, n, err_word);
      out[pq * n + k] = on_frontier(plane, n, q, k, nq, nk) ? 1 : 0;
    }
  }
}

__global__ void __launch_bounds__(kCellThreads) candidate_scatter_kernel(DirectionalArgs a) {
  const int n = a.n;
  // One CTA per (plane, q) row at a time, threads across k (no per-cell
  // divisions; the row's Q neighbours are loaded once).
  const int64_t rows = a.planes * n;
  for (int64_t pq = blockIdx.x; pq < rows; pq += gridDim.x) {
    const int q = static_cast<int>(pq % n);
    const int64_t p0 = (pq - q) * n;
    const uint8_t* prev = a.prev + p0;
    const float* mass = a.mass + p0;
    const int4 nq = load_neighbors(a.neighbors, q, n, a.err_word);
    for (int k = threadIdx.x; k < n; k += kCellThreads) {
      const int64_t c = pq * n + k;
      const int4 nk = load_neighbors(a.neighbors, k, n, a.err_word);
      const bool front = a.prev_frontier != nullptr ? a.prev_frontier[c] != 0
                                                    : on_frontier(prev, n, q, k, nq, nk);
      if (!front) continue;
      const float floor_value = __fmul_rn(mass[static_cast<size_t>(q) * n + k], a.min_ratio);
      // Along Q: neighbour rows t of this column; along K: neighbour columns t
      // of this row.  A neighbour counts when it exists and is unselected;
      // the first of equal maxima wins.
      float best_q = -INFINITY, best_k = -INFINITY;
      int tgt_q = max(nq.x, 0), tgt_k = max(nk.x, 0);
#pragma unroll
      for (int d = 0; d < 4; ++d) {
        const int tq = nb_at(nq, d);
        const float vq = (tq >= 0 && !prev[static_cast<size_t>(tq) * n + k])
                             ? mass[static_cast<size_t>(tq) * n + k] : -INFINITY;
        if (d == 0 || vq > best_q) {
          if (d != 0) tgt_q = tq;
          best_q = vq;
        }
        const int tk = nb_at(nk, d);
        const float vk = (tk >= 0 && !prev[static_cast<size_t>(q) * n + tk])
                             ? mass[static_cast<size_t>(q) * n + tk] : -INFINITY;
        if (d == 0 || vk > best_k) {
          if (d != 0) tgt_k = tk;
          best_k = vk;
        }
      }
      const bool elig_q = isfinite(best_q) && best_q >= floor_value;
      const bool elig_k = isfinite(best_k) && best_k >= floor_value;
      uint8_t* cand = a.candidates + p0;
      if ((a.expand & kExpandQ) && elig_q) cand[static_cast<size_t>(tgt_q) * n + k] = 1;
      if ((a.expand & kExpandK) && elig_k) cand[static_cast<size_t>(q) * n + tgt_k] = 1;
      if ((a.expand & kExpandJoint) && elig_q && elig_k)
        cand[static_cast<size_t>(tgt_q) * n + tgt_k] = 1;
    }
  }
}

__device__ int block_sum(int local, int* s_acc) {
  if (threadIdx.x == 0) *s_acc = 0;
  __syncthreads();
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) local += __shfl_xor_sync(0xffffffffu, local, off);
  if ((threadIdx.x & 31) == 0) atomicAdd(s_acc, local);
  __syncthreads();
  const int total = *s_acc;
  __syncthreads();
  return total;
}

__global__ void __launch_bounds__(kSelThreads) directional_select_kernel(DirectionalArgs a,
                                                                         int np) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int n = a.n;
  uint64_t* keys = reinterpret_cast<uint64_t*>(smem);          // [np]
  float* vals = reinterpret_cast<float*>(keys + np);           // [n] mass
  float* score = vals + n;                                     // [n]
  uint8_t* fprev = reinterpret_cast<uint8_t*>(score + n);      // [n] each
  uint8_t* fcand = fprev + n;
  uint8_t* fpool = fcand + n;
  uint8_t* fexpl = fpool + n;
  uint8_t* froute = fexpl + n;
  __shared__ int s_acc;
  __shared__ float s_row_scale;

  const int tid = threadIdx.x;
  const int64_t row = blockIdx.x;
  const size_t base = static_cast<size_t>(row) * n;

  // ---- pool = prev | (candidates & ~prev) ---------------------------------
  int prev_local = 0;
  for (int i = tid; i < n; i += kSelThreads) {
    vals[i] = a.mass[base + i];
    const uint8_t p = a.prev[base + i] ? 1 : 0;
    const uint8_t c = (a.candidates[base + i] && !p) ? 1 : 0;
    fprev[i] = p;
    fcand[i] = c;
    fpool[i] = p | c;
    fexpl[i] = 0;
    prev_local += p;
  }
  const int prev_count = block_sum(prev_local, &s_acc);

  // ---- exploration: the explore_count highest masses outside the pool -----
  if (a.explore_count > 0) {
    for (int i = tid; i < n; i += kSelThreads) score[i] = fpool[i] ? -INFINITY : vals[i];
    __syncthreads();
    sort_row_desc(score, n, np, keys);
    mark_first_desc(score, n, a.explore_count, keys, fexpl);
    for (int i = tid; i < n; i += kSelThreads) fpool[i] |= fexpl[i];
  }
  int pool_local = 0;
  for (int i = tid; i < n; i += kSelThreads) pool_local += fpool[i];
  const int pool_count = block_sum(pool_local, &s_acc);

  // ---- score = mass + p*mean(mass)*prev [+ bonus*mean(mass)*candidates] ----
  if (tid < 32) {
    const float sum = torch_cpu_row_sum(vals, n);
    if (tid == 0) s_row_scale = __fdiv_rn(sum, static_cast<float>(n));
  }
  __syncthreads();
  const float bump = __fmul_rn(s_row_scale, a.persistence);
  const float cbump = __fmul_rn(s_row_scale, a.candidate_bonus);
  for (int i = tid; i < n; i += kSelThreads) {
    float s = __fadd_rn(vals[i], __fmul_rn(bump, fprev[i] ? 1.f : 0.f));
    if (a.candidate_bonus != 0.f) s = __fadd_rn(s, __fmul_rn(cbump, fcand[i] ? 1.f : 0.f));
    score[i] = fpool[i] ? s : -INFINITY;
  }
  __syncthreads();

  // ---- fixed budget: ceil(#prev * scale) in [1, cap], at most the pool -----
  int count = static_cast<int>(ceilf(__fmul_rn(static_cast<float>(prev_count), a.budget_scale)));
  count = min(max(count, 1), a.cap);
  count = max(min(count, pool_count), 1);
  sort_row_desc(score, n, np, keys);
  mark_first_desc(score, n, count, keys, froute);

  // ---- outputs before the sink, then the sink and the CSR ----------------
  for (int i = tid; i < n; i += kSelThreads) {
    const uint8_t r = froute[i] & fpool[i];
    a.candidates[base + i] = fcand[i];
    if (a.exploration != nullptr) a.exploration[base + i] = fexpl[i];
    if (a.dropped != nullptr) a.dropped[base + i] = fprev[i] & (r ^ 1);
    if (a.added != nullptr) a.added[base + i] = r & (fprev[i] ^ 1);
    froute[i] = (r || i < a.sink_blocks) ? 1 : 0;
  }
  __syncthreads();
  write_csr_row(froute, n, base, a.indices, a.route_out,
                a.counts != nullptr ? a.counts + row : nullptr,
                a.kept != nullptr ? a.kept + row / a.rows_per_group : nullptr);
}

// Warp-per-row version of directional_select_kernel for n <= 512 (same
// outputs): the two selections use the register sort of route_common.cuh.
constexpr int kDirWarps = 4;  // rows per CTA

struct DirWarpSmem {
  SortPair pairs[kWarpSelMaxCols];                      // tie replay scratch
  float vals[kWarpSelMaxCols + kWarpSelMaxCols / 16];   // mass at vidx(i)
  float score[kWarpSelMaxCols + kWarpSelMaxCols / 16];  // selection score at vidx(i)
  uint8_t fprev[kWarpSelMaxCols], fcand[kWarpSelMaxCols], fpool[kWarpSelMaxCols],
      fexpl[kWarpSelMaxCols], froute[kWarpSelMaxCols];
};

template <int ITEMS>
__global__ void __launch_bounds__(kDirWarps * 32) directional_select_warp_kernel(
    DirectionalArgs a) {
  __shared__ DirWarpSmem smem_all[kDirWarps];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n = a.n;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kDirWarps + warp;
  if (row >= a.planes * n) return;  // warp-uniform; no CTA barrier below
  DirWarpSmem& sm = smem_all[warp];
  const size_t base = static_cast<size_t>(row) * n;
  float* vals = sm.vals;
  float* score = sm.score;

  // ---- pool = prev | (candidates & ~prev) ---------------------------------
  int prev_local = 0;
  for (int i = lane; i < n; i += 32) {
    vals[vidx(i)] = a.mass[base + i];
    const uint8_t p = a.prev[base + i] ? 1 : 0;
    const uint8_t c = (a.candidates[base + i] && !p) ? 1 : 0;
    sm.fprev[i] = p;
    sm.fcand[i] = c;
    sm.fpool[i] = p | c;
    sm.fexpl[i] = 0;
    prev_local += p;
  }
  const int prev_count = __reduce_add_sync(kFull, prev_local);
  __syncwarp();

  // ---- exploration: the explore_count highest masses outside the pool -----
  if (a.explore_count > 0) {
    for (int i = lane; i < n; i += 32) score[vidx(i)] = sm.fpool[i] ? -INFINITY : vals[vidx(i)];
    __syncwarp();
    warp_mark_first_desc<ITEMS>(score, n, a.explore_count, sm.pairs, sm.fexpl);
    for (int i = lane; i < n; i += 32) sm.fpool[i] |= sm.fexpl[i];
    __syncwarp();
  }
  int pool_local = 0;
  for (int i = lane; i < n; i += 32) pool_local += sm.fpool[i];
  const int pool_count = __reduce_add_sync(kFull, pool_local);

  // ---- score = mass + p*mean(mass)*prev [+ bonus*mean(mass)*candidates] ----
  const float sum = torch_cpu_sum([vals](int i) { return vals[vidx(i)]; }, n);
  const float row_scale = __fdiv_rn(sum, static_cast<float>(n));
  const float bump = __fmul_rn(row_scale, a.persistence);
  const float cbump = __fmul_rn(row_scale, a.candidate_bonus);
  __syncwarp();
  for (int i = lane; i < n; i += 32) {
    float s = __fadd_rn(vals[vidx(i)], __fmul_rn(bump, sm.fprev[i] ? 1.f : 0.f));
    if (a.candidate_bonus != 0.f) s = __fadd_rn(s, __fmul_rn(cbump, sm.fcand[i] ? 1.f : 0.f));
    score[vidx(i)] = sm.fpool[i] ? s : -INFINITY;
  }
  __syncwarp();

  // ---- fixed budget: ceil(#prev * scale) in [1, cap], at most the pool -----
  int count = static_cast<int>(ceilf(__fmul_rn(static_cast<float>(prev_count), a.budget_scale)));
  count = min(max(count, 1), a.cap);
  count = max(min(count, pool_count), 1);
  warp_mark_first_desc<ITEMS>(score, n, count, sm.pairs, sm.froute);

  // ---- outputs before the sink, then the sink and the CSR ----------------
  for (int i = lane; i < n; i += 32) {
    const uint8_t r = sm.froute[i] & sm.fpool[i];
    const uint8_t p = sm.fprev[i];
    a.candidates[base + i] = sm.fcand[i];
    if (a.exploration != nullptr) a.exploration[base + i] = sm.fexpl[i];
    if (a.dropped != nullptr) a.dropped[base + i] = p & (r ^ 1);
    if (a.added != nullptr) a.added[base + i] = r & (p ^ 1);
    sm.froute[i] = (r || i < a.sink_blocks) ? 1 : 0;
  }
  __syncwarp();
  warp_write_csr_row(sm.froute, n, base, a.indices, a.route_out,
                     a.counts != nullptr ? a.counts + row : nullptr,
                     a.kept != nullptr ? a.kept + row / a.rows_per_group : nullptr);
}

template <int ITEMS>
cudaError_t launch_directional_warp(const DirectionalArgs& a, int64_t rows, cudaStream_t stream) {
  const int64_t ctas = (rows + kDirWarps - 1) / kDirWarps;
  directional_select_warp_kernel<ITEMS>
      <<<static_cast<unsigned>(ctas), kDirWarps * 32, 0, stream>>>(a);
  return cudaGetLastError();
}

// Row-strided grid: one CTA per (plane, q) row, at most 8 CTAs per SM.
unsigned row_grid(int64_t rows, int num_sms) {
  const int64_t cap = static_cast<int64_t>(num_sms) * 8;
  return static_cast<unsigned>(rows < cap ? (rows > 0 ? rows : 1) : cap);
}

}  // namespace

cudaError_t launch_frontier_mask(const uint8_t* route, const int32_t* neighbors, int64_t planes,
                                 int32_t n, uint8_t* frontier, int* err_word,
                                 cudaStream_t stream, int num_sms) {
  const int64_t cells = planes * n * static_cast<int64_t>(n);
  if (cells == 0) return cudaSuccess;
  frontier_kernel<<<row_grid(planes * n, num_sms), kCellThreads, 0, stream>>>(route, neighbors, planes,
                                                                          n, frontier, err_word);
  return cudaGetLastError();
}

cudaError_t launch_directional_update(const DirectionalArgs& a, cudaStream_t stream,
                                      int num_sms) {
  const int64_t rows = a.planes * a.n;
  if (rows == 0) return cudaSuccess;
  if (a.n <= 0 || a.n > kMaxCols) return cudaErrorInvalidValue;
  candidate_scatter_kernel<<<row_grid(rows, num_sms), kCellThreads, 0, stream>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  if (a.n <= 32) return launch_directional_warp<1>(a, rows, stream);
  if (a.n <= 64) return launch_directional_warp<2>(a, rows, stream);
  if (a.n <= 128) return launch_directional_warp<4>(a, rows, stream);
  if (a.n <= 256) return launch_directional_warp<8>(a, rows, stream);
  if (a.n <= kWarpSelMaxCols) return launch_directional_warp<16>(a, rows, stream);
  int np = 1;
  while (np < a.n) np <<= 1;
  const size_t smem = static_cast<size_t>(np) * 8 + static_cast<size_t>(a.n) * 13 + 16;
  if (smem > 48 * 1024) {
    e = cudaFuncSetAttribute(directional_select_kernel,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  directional_select_kernel<<<static_cast<unsigned>(rows), kSelThreads, smem, stream>>>(a, np);
  return cudaGetLastError();
}

}  // namespace bsa
