// (c) Spatial reorder: out[t][b][i][:] = src[t][b][perm[i]][:] for up to three
// tensors sharing one permutation.  Pack (Q/K/V into Morton order) and unpack
// (output back to raster order, with the inverse permutation) are both this
// gather, so every store is a coalesced full row.  With a destination row map
// the same kernel writes out[t][b][dst_rows[i]] instead (the head-parallel
// exchange uses it to lay rows out for the all-to-all).
//
// Reference semantics: attention_backends/spatial.py:82-93 (index_select on
// axis 1) and the fused Triton gather attention_backends/layout_ops.py:21-52,
// 86-125.
#include "bsa_kernels.h"

namespace bsa {
namespace {

constexpr int kReorderWarps = 8;
constexpr int kUnroll = 4;

struct ReorderArgs {
  const uint8_t* src[3];
  uint8_t* dst[3];
  const int32_t* perm;
  const int32_t* dst_rows;  // destination row of each output index, or null (row i)
  int64_t batch;
  int64_t tokens_out;       // output indices per batch element
  int64_t tokens_in;
  int64_t tokens_dst;       // destination rows per batch element
  int64_t row_bytes;
  int64_t rows_per_tensor;  // batch * tokens_out
  int n_tensors;
  int* err_word;
};

// One warp copies one output row per iteration; each lane moves kUnroll
// vectors per step so several loads are in flight before the stores.
template <typename Vec>
__global__ void __launch_bounds__(kReorderWarps * 32)
    reorder_rows_kernel(const __grid_constant__ ReorderArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t warp_global = (static_cast<int64_t>(blockIdx.x) * kReorderWarps) + (threadIdx.x >> 5);
  const int64_t total = a.rows_per_tensor * a.n_tensors;
  const int64_t nvec = a.row_bytes / static_cast<int64_t>(sizeof(Vec));
  const int64_t warp_stride = static_cast<int64_t>(gridDim.x) * kReorderWarps;
  for (int64_t r = warp_global; r < total; r += warp_stride) {
    const int t = static_cast<int>(r / a.rows_per_tensor);
    const int64_t rr = r - static_cast<int64_t>(t) * a.rows_per_tensor;
    const int64_t b = rr / a.tokens_out;
    const int64_t i = rr - b * a.tokens_out;
    int64_t s = __ldg(a.perm + i);
    if (s < 0 || s >= a.tokens_in) {
      if (lane == 0 && a.err_word) atomicOr(a.err_word, kErrBadRoute);
      continue;
    }
    int64_t d = i;
    if (a.dst_rows != nullptr) {
      d = __ldg(a.dst_rows + i);
      if (d < 0 || d >= a.tokens_dst) {
        if (lane == 0 && a.err_word) atomicOr(a.err_word, kErrBadRoute);
        continue;
      }
    }
    const uint8_t* src_base = t == 0 ? a.src[0] : (t == 1 ? a.src[1] : a.src[2]);
    uint8_t* dst_base = t == 0 ? a.dst[0] : (t == 1 ? a.dst[1] : a.dst[2]);
    const Vec* src = reinterpret_cast<const Vec*>(src_base + (b * a.tokens_in + s) * a.row_bytes);
    Vec* dst = reinterpret_cast<Vec*>(dst_base + (b * a.tokens_dst + d) * a.row_bytes);
    int64_t v = lane;
    for (; v + 32 * (kUnroll - 1) < nvec; v += 32 * kUnroll) {
      Vec tmp[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) tmp[u] = __ldcs(src + v + 32 * u);
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) dst[v + 32 * u] = tmp[u];
    }
    for (; v < nvec; v += 32) dst[v] = __ldcs(src + v);
  }
}

// Head-parallel input exchange by pulls over peer memory: packed row i of
// tensor x (Q, K, V) is token t = perm[i], held by rank p = t / peer_tokens
// at its token t - p * peer_tokens; the row's bytes for this call's heads are
// read from rank p's input shard (mapped into this process) and stored to
// dst[x] row i.  One warp per row, 16-byte vectors.
struct PullArgs {
  const uint8_t* src[kMaxPeers];  // rank p's input shard
  uint8_t* dst[3];
  const int32_t* perm;            // or null: row i is token i
  int64_t tokens;
  int64_t peer_tokens;
  int64_t src_row_bytes;          // between consecutive tokens of a shard
  int64_t src_tensor_bytes;       // between Q, K and V of a shard
  int64_t src_offset;             // this call's heads within a token's row
  int64_t row_bytes;              // bytes pulled per row
  int n_peers;
  int* err_word;
};

__global__ void __launch_bounds__(kReorderWarps * 32)
    pull_rows_kernel(const __grid_constant__ PullArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t warp_global = (static_cast<int64_t>(blockIdx.x) * kReorderWarps) + (threadIdx.x >> 5);
  const int64_t total = 3 * a.tokens;
  const int64_t nvec = a.row_bytes / 16;
  const int64_t warp_stride = static_cast<int64_t>(gridDim.x) * kReorderWarps;
  for (int64_t r = warp_global; r < total; r += warp_stride) {
    const int x = static_cast<int>(r / a.tokens);
    const int64_t i = r - static_cast<int64_t>(x) * a.tokens;
    const int64_t t = a.perm != nullptr ? static_cast<int64_t>(__ldg(a.perm + i)) : i;
    const int64_t p = t >= 0 ? t / a.peer_tokens : -1;
    if (t < 0 || t >= a.tokens || p >= a.n_peers) {
      if (lane == 0 && a.err_word) atomicOr(a.err_word, kErrBadRoute);
      continue;
    }
    const int64_t lt = t - p * a.peer_tokens;
    const uint4* src = reinterpret_cast<const uint4*>(a.src[p] + x * a.src_tensor_bytes +
                                                      lt * a.src_row_bytes + a.src_offset);
    uint4* dst = reinterpret_cast<uint4*>((x == 0 ? a.dst[0] : (x == 1 ? a.dst[1] : a.dst[2])) +
                                          i * a.row_bytes);
    int64_t v = lane;
    for (; v + 32 * (kUnroll - 1) < nvec; v += 32 * kUnroll) {
      uint4 tmp[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) tmp[u] = __ldcg(src + v + 32 * u);
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) dst[v + 32 * u] = tmp[u];
    }
    for (; v < nvec; v += 32) dst[v] = __ldcg(src + v);
  }
}

}  // namespace

cudaError_t launch_pull_rows(const void* const* peers, int n_peers, int64_t peer_tokens,
                             int64_t src_row_bytes, int64_t src_tensor_bytes,
                             int64_t src_offset, const int32_t* perm, int64_t tokens,
                             int64_t row_bytes, void* const* dst, int* err_word,
                             cudaStream_t stream, int num_sms) {
  if (n_peers < 1 || n_peers > kMaxPeers || peer_tokens <= 0 || tokens <= 0 ||
      row_bytes <= 0 || (row_bytes & 15) || (src_row_bytes & 15) || (src_tensor_bytes & 15) ||
      (src_offset & 15) || peer_tokens * n_peers != tokens)
    return cudaErrorInvalidValue;
  PullArgs a{};
  for (int p = 0; p < n_peers; ++p) {
    if (peers[p] == nullptr || (reinterpret_cast<uintptr_t>(peers[p]) & 15))
      return cudaErrorInvalidValue;
    a.src[p] = static_cast<const uint8_t*>(peers[p]);
  }
  for (int x = 0; x < 3; ++x) {
    if (dst[x] == nullptr || (reinterpret_cast<uintptr_t>(dst[x]) & 15))
      return cudaErrorInvalidValue;
    a.dst[x] = static_cast<uint8_t*>(dst[x]);
  }
  a.perm = perm;
  a.tokens = tokens;
  a.peer_tokens = peer_tokens;
  a.src_row_bytes = src_row_bytes;
  a.src_tensor_bytes = src_tensor_bytes;
  a.src_offset = src_offset;
  a.row_bytes = row_bytes;
  a.n_peers = n_peers;
  a.err_word = err_word;
  int64_t blocks = (3 * tokens + kReorderWarps - 1) / kReorderWarps;
  const int64_t cap = static_cast<int64_t>(num_sms) * 16;
  if (blocks > cap) blocks = cap;
  pull_rows_kernel<<<static_cast<unsigned>(blocks), kReorderWarps * 32, 0, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_reorder_rows(int n_tensors, const void* const* src, void* const* dst,
                                const int32_t* perm, int64_t batch, int64_t tokens_out,
                                int64_t tokens_in, int64_t row_bytes, int* err_word,
                                cudaStream_t stream, int num_sms, const int32_t* dst_rows,
                                int64_t tokens_dst) {
  ReorderArgs a{};
  a.dst_rows = dst_rows;
  a.tokens_dst = dst_rows != nullptr ? tokens_dst : tokens_out;
  uintptr_t align_bits = static_cast<uintptr_t>(row_bytes);
  for (int t = 0; t < n_tensors; ++t) {
    a.src[t] = static_cast<const uint8_t*>(src[t]);
    a.dst[t] = static_cast<uint8_t*>(dst[t]);
    align_bits |= reinterpret_cast<uintptr_t>(src[t]) | reinterpret_cast<uintptr_t>(dst[t]);
  }
  a.perm = perm;
  a.batch = batch;
  a.tokens_out = tokens_out;
  a.tokens_in = tokens_in;
  a.row_bytes = row_bytes;
  a.rows_per_tensor = batch * tokens_out;
  a.n_tensors = n_tensors;
  a.err_word = err_word;
  const int64_t rows = a.rows_per_tensor * n_tensors;
  if (rows == 0) return cudaSuccess;
  // Enough warps to keep every SM's load queue full; each warp loops.
  int64_t blocks = (rows + kReorderWarps - 1) / kReorderWarps;
  const int64_t cap = static_cast<int64_t>(num_sms) * 16;
  if (blocks > cap) blocks = cap;
  const dim3 grid(static_cast<unsigned>(blocks));
  const dim3 block(kReorderWarps * 32);
  if ((align_bits & 15) == 0) {
    reorder_rows_kernel<uint4><<<grid, block, 0, stream>>>(a);
  } else if ((align_bits & 7) == 0) {
    reorder_rows_kernel<uint2><<<grid, block, 0, stream>>>(a);
  } else if ((align_bits & 3) == 0) {
    reorder_rows_kernel<uint32_t><<<grid, block, 0, stream>>>(a);
  } else if ((align_bits & 1) == 0) {
    reorder_rows_kernel<uint16_t><<<grid, block, 0, stream>>>(a);
  } else {
    reorder_rows_kernel<uint8_t><<<grid, block, 0, stream>>>(a);
  }
  return cudaGetLastError();
}

}  // namespace bsa
