// C ABI of libbsa.so (declared in include/bsa.h): argument validation, TMA
// tensor-map encoding and kernel launch.  No entry point allocates memory or
// synchronises the stream.
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <atomic>
#include <mutex>
#include <string>

#include "../../include/bsa.h"
#include "bsa_kernels.h"

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* where) {
  return fail(BSA_ERR_CUDA, "%s: %s (%s)", where, cudaGetErrorName(e), cudaGetErrorString(e));
}

int ok() {
  g_last_error.clear();
  return BSA_OK;
}

int sm_count() {
  static std::atomic<int> cached[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev >= 0 && dev < 64) {
    const int c = cached[dev].load(std::memory_order_relaxed);
    if (c > 0) return c;
  }
  int n = 148;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (dev >= 0 && dev < 64) cached[dev].store(n, std::memory_order_relaxed);
  return n;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 4-D bf16 tensor map over a [B, T, H, D] tensor with element strides
// (sb, st, sh), D contiguous.  Box: 64 features x `rows` tokens x 1 head x 1
// batch, 128-byte swizzle, zero fill out of bounds.  Dimensions are ordered by
// increasing stride: (D, H, T, B) when sh <= st, else (D, T, H, B); `t_major`
// reports the second case (coordinate order (d, t, h, b)).
int encode_bhtd(CUtensorMap* map, const void* ptr, int64_t B, int64_t T, int64_t H, int64_t D,
                int64_t sb, int64_t st, int64_t sh, int rows, bool* t_major) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return fail(BSA_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  if ((reinterpret_cast<uintptr_t>(ptr) & 15) != 0)
    return fail(BSA_ERR_INVALID_ARGUMENT, "tensor base address must be 16-byte aligned");
  if (((sb * 2) & 15) || ((st * 2) & 15) || ((sh * 2) & 15))
    return fail(BSA_ERR_INVALID_ARGUMENT,
                "token/head/batch strides must be multiples of 8 elements (16 bytes)");
  *t_major = st < sh;
  cuuint64_t dims[4], strides[3];
  dims[0] = static_cast<cuuint64_t>(D);
  if (!*t_major) {
    dims[1] = H; dims[2] = T;
    strides[0] = sh * 2; strides[1] = st * 2;
  } else {
    dims[1] = T; dims[2] = H;
    strides[0] = st * 2; strides[1] = sh * 2;
  }
  dims[3] = B;
  strides[2] = sb * 2;
  if (B == 1) strides[2] = strides[1] * dims[2];  // unused; keep it well-formed
  cuuint32_t box[4] = {64u, 1u, static_cast<cuuint32_t>(rows), 1u};
  if (*t_major) { box[1] = static_cast<cuuint32_t>(rows); box[2] = 1u; }
  cuuint32_t estr[4] = {1u, 1u, 1u, 1u};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(ptr), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(BSA_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return BSA_OK;
}

}  // namespace

namespace {

// Checks and tensor maps shared by the two sampled-mass entry points.
int sampled_mass_setup(const void* sampled_q, const void* sampled_k, int64_t batch,
                       int64_t heads, int32_t q_blocks, int32_t samples, int32_t head_dim,
                       const float* block_bias, float scale, int32_t round_bf16, float* mass,
                       int32_t* err_word, CUtensorMap* tq, CUtensorMap* tk, bsa::MassArgs* a) {
  if (sampled_q == nullptr || sampled_k == nullptr || block_bias == nullptr || mass == nullptr ||
      err_word == nullptr)
    return fail(BSA_ERR_INVALID_ARGUMENT, "null pointer argument");
  if (head_dim != 128) return fail(BSA_ERR_UNSUPPORTED, "head_dim must be 128 (got %d)", head_dim);
  if (samples != 1 && samples != 2 && samples != 4 && samples != 8 && samples != 16 &&
      samples != 32)
    return fail(BSA_ERR_UNSUPPORTED, "samples must be a power of two <= 32 (got %d)", samples);
  if (q_blocks <= 0 || q_blocks > 4096)
    return fail(BSA_ERR_UNSUPPORTED, "q_blocks must be in [1, 4096] (got %d)", q_blocks);
  if (batch <= 0 || heads <= 0 || batch > 65535 || heads > 65535)
    return fail(BSA_ERR_INVALID_ARGUMENT, "bad batch/heads");
  const int64_t n_rows = static_cast<int64_t>(q_blocks) * samples;
  bool tm = false;
  int rc = encode_bhtd(tq, sampled_q, batch, n_rows, heads, head_dim, n_rows * heads * head_dim,
                       heads * head_dim, head_dim, 128, &tm);
  if (rc != BSA_OK) return rc;
  rc = encode_bhtd(tk, sampled_k, batch, n_rows, heads, head_dim, n_rows * heads * head_dim,
                   heads * head_dim, head_dim, 128, &tm);
  if (rc != BSA_OK) return rc;
  if (tm) return fail(BSA_ERR_INVALID_ARGUMENT, "sampled tensors must be [B, N, H, D] contiguous");
  *a = bsa::MassArgs{};
  a->batch = batch;
  a->heads = heads;
  a->n_rows = n_rows;
  a->samples = samples;
  a->q_blocks = q_blocks;
  a->scale = scale;
  a->round_bf16 = round_bf16;
  a->block_bias = block_bias;
  a->mass_scale = 1.0f / static_cast<float>(samples);
  a->mass = mass;
  a->err_word = err_word;
  return BSA_OK;
}

}  // namespace

extern "C" {

int bsa_version(void) { return 10000; }

const char* bsa_last_error(void) { return g_last_error.c_str(); }

int bsa_reorder_rows(int32_t n_tensors, const void* const* src, void* const* dst,
                     const int32_t* perm, int64_t batch, int64_t tokens_out, int64_t tokens_in,
                     int64_t row_bytes, int32_t* err_word, void* stream) {
  if (n_tensors < 1 || n_tensors > 3)
    return fail(BSA_ERR_INVALID_ARGUMENT, "n_tensors must be 1, 2 or 3");
  if (src == nullptr || dst == nullptr || perm == nullptr)
    return fail(BSA_ERR_INVALID_ARGUMENT, "null pointer argument");
  for (int t = 0; t < n_tensors; ++t)
    if (src[t] == nullptr || dst[t] == nullptr)
      return fail(BSA_ERR_INVALID_ARGUMENT, "null tensor pointer %d", t);
  if (batch < 0 || tokens_out < 0 || tokens_in < 0 || row_bytes <= 0)
    return fail(BSA_ERR_INVALID_ARGUMENT, "negative size or empty row");
  cudaError_t e = bsa::launch_reorder_rows(n_tensors, src, dst, perm, batch, tokens_out,
                                           tokens_in, row_bytes, err_word,
                                           static_cast<cudaStream_t>(stream), sm_count());
  if (e != cudaSuccess) return cuda_fail(e, "bsa_reorder_rows launch");
  return ok();
}

int bsa_gather_scatter_rows(int32_t n_tensors, const void* const* src, void* const* dst,
                            const int32_t* src_rows, const int32_t* dst_rows, int64_t batch,
                            int64_t rows, int64_t tokens_in, int64_t tokens_dst,
                            int64_t row_bytes, int32_t* err_word, void* stream) {
  if (n_tensors < 1 || n_tensors > 3)
    return fail(BSA_ERR_INVALID_ARGUMENT, "n_tensors must be 1, 2 or 3");
  if (src == nullptr || dst == nullptr || src_rows == nullptr || dst_rows == nullptr)
    return fail(BSA_ERR_INVALID_ARGUMENT, "null pointer argument");
  for (int t = 0; t < n_tensors; ++t)
    if (src[t] == nullptr || dst[t] == nullptr)
      return fail(BSA_ERR_INVALID_ARGUMENT, "null tensor pointer %d", t);
  if (batch < 0 || rows < 0 || tokens_in < 0 || tokens_dst < 0 || row_bytes <= 0)
    return fail(BSA_ERR_INVALID_ARGUMENT, "negative size or empty row");
  cudaError_t e = bsa::launch_reorder_rows(n_tensors, src, dst, src_rows, batch, rows, tokens_in,
                                           row_bytes, err_word, static_cast<cudaStream_t>(stream),
                                           sm_count(), dst_rows, tokens_dst);
  if (e != cudaSuccess) return cuda_fail(e, "bsa_gather_scatter_rows launch");
  return ok();
}

int bsa_pack_boolean_rows(const uint8_t* route, int64_t rows, int32_t cols, int32_t* counts,
                          int32_t* indices, void* stream) {
  if (route == nullptr || counts == nullptr || indices == nullptr)
    return fail(BSA_ERR_INVALID_ARGUMENT, "null pointer argument");
  if (rows < 0 || cols <= 0 || cols > 4096)
    return fail(BSA_ERR_UNSUPPORTED, "cols must be in [1, 4096] (got %d)", cols);
  bsa::SelectArgs a{};
  a.route_in = route;
  a.rows = rows;
  a.cols = cols;
  a.rows_per_group = 1;
  a.counts = counts;
  a.indices = indices;
  cudaError_t e = bsa::launch_route_select(a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "bsa_pack_boolean_rows launch");
  return ok();
}

int bsa_route_select(const float* mass, const uint8_t* prev, int64_t rows, int32_t cols,
                     int32_t rows_per_group, float persistence, float target,
                     int32_t max_blocks, int32_t sink_blocks, uint8_t* route_out,
                     int32_t* counts, int32_t* indices, uint64_t* kept, void* stream) {
  if (mass == nullptr) return fail(BSA_ERR_INVALID_ARGUMENT, "mass is null");
  if (rows < 0 || cols <= 0 || cols > 4096)
    return fail(BSA_ERR_UNSUPPORTED, "cols must be in [1, 4096] (got %d)", cols);
  if (max_blocks < 1 || max_blocks > cols)
    return fail(BSA_ERR_INVALID_ARGUMENT, "max_blocks must be in [1, cols] (got %d)", max_blocks);
  if (!(target > 0.f && target <= 1.f))
    return fail(BSA_ERR_INVALID_ARGUMENT, "mass_target must be in (0, 1]");
  if (persistence < 0.f) return fail(BSA_ERR_INVALID_ARGUMENT, "persistence must be >= 0");
  if (kept != nullptr && (rows_per_group <= 0 || rows % rows_per_group != 0))
    return fail(BSA_ERR_INVALID_ARGUMENT, "rows must be a multiple of rows_per_group");
  bsa::SelectArgs a{};
  a.mass = mass;
  a.prev = prev;
  a.persistence = persistence;
  a.target = target;
  a.cap = max_blocks;
  a.sink_blocks = sink_blocks < 0 ? 0 : sink_blocks;
  a.rows = rows;
  a.cols = cols;
  a.rows_per_group = rows_per_group > 0 ? rows_per_group : 1;
  a.route_out = route_out;
  a.counts = counts;
  a.indices = indices;
  a.kept = reinterpret_cast<unsigned long long*>(kept);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (kept != nullptr) {
    cudaError_t e = cudaMemsetAsync(kept, 0, sizeof(uint64_t) * (rows / a.rows_per_group), s);
    if (e != cudaSuccess) return cuda_fail(e, "bsa_route_select memset");
  }
  cudaError_t e = bsa::launch_route_select(a, s);
  if (e != cudaSuccess) return cuda_fail(e, "bsa_route_select launch");
  return ok();
}

int bsa_qkv_prologue(const void* q_proj, const void* k_proj, const void* v_proj, int64_t batch,
                     int64_t tokens, int64_t heads, int32_t head_dim, int64_t in_stride_b,
                     int64_t in_stride_t, int32_t norm_q, int32_t norm_k,
                     const float* norm_q_weight, const float* norm_k_weight, float eps,
                     const float* rope_cos, const float* rope_sin, const int32_t* perm,
                     void* q_out, void* k_out, void* v_out, int32_t* err_word, void* stream) {
  if (q_proj == nullptr || k_proj == nullptr || v_proj == nullptr || q_out == nullptr ||
      k_out == nullptr || v_out == nullptr || err_word == nullptr)
    return fail(BSA_ERR_INVALID_ARGUMENT, "null pointer argument");
  if (batch < 0 || tokens < 0 || heads <= 0 || head_dim <= 0 || head_dim % 8 != 0 ||
      heads * head_dim > (1 << 20))
    return fail(BSA_ERR_INVALID_ARGUMENT, "bad batch/tokens/heads/head_dim (head_dim %% 8 == 0)");
  if ((rope_cos == nullptr) != (rope_sin == nullptr))
    return fail(BSA_ERR_INVALID_ARGUMENT, "rope_cos and rope_sin go together");
  const void* ptrs[] = {q_proj, k_proj, v_proj, q_out, k_out, v_out, rope_cos, rope_sin,
                        norm_q_weight, norm_k_weight};
  for (const void* p : ptrs)
    if (reinterpret_cast<uintptr_t>(p) & 15)
      return fail(BSA_ERR_INVALID_ARGUMENT, "tensors must be 16-byte aligned");
  if ((in_stride_b * 2) % 16 || (in_stride_t * 2) % 16)
    return fail(BSA_ERR_INVALID_ARGUMENT, "row strides must be multiples of 8 elements");
  bsa::PrologueArgs a{};
  a.q_in = static_cast<const __nv_bfloat16*>(q_proj);
  a.k_in = static_cast<const __nv_bfloat16*>(k_proj);
  a.v_in = static_cast<const __nv_bfloat16*>(v_proj);
  a.batch = batch;
  a.tokens = tokens;
  a.heads = static_cast<int32_t>(heads);
  a.head_dim = head_dim;
  a.in_stride_b = in_stride_b;
  a.in_stride_t = in_stride_t;
  a.norm_q = norm_q != 0;
  a.norm_k = norm_k != 0;
  a.weight_q = norm_q_weight;
  a.weight_k = norm_k_weight;
  a.eps = eps;
  a.rope_cos = rope_cos;
  a.rope_sin = rope_sin;
  a.perm = perm;
  a.q_out = static_cast<__nv_bfloat16*>(q_out);
  a.k_out = static_cast<__nv_bfloat16*>(k_out);
  a.v_out = static_cast<__nv_bfloat16*>(v_out);
  a.err_word = err_word;
  cudaError_t e = bsa::launch_qkv_prologue(a, static_cast<cudaStream_t>(stream), sm_count());
  if (e != cudaSuccess) return cuda_fail(e, "bsa_qkv_prologue launch");
  return ok();
}

int bsa_frontier_mask(const uint8_t* route, const int32_t* neighbors, int64_t planes,
                      int32_t blocks, uint8_t* frontier, int32_t* err_word, void* stream) {
  if (route == nullptr || neighbors == nullptr || frontier == nullptr)
    return fail(BSA_ERR_INVALID_ARGUMENT, "route, neighbors and frontier must not be null");
  if (planes < 0 || blocks <= 0 || blocks > 4096)
    return fail(BSA_ERR_UNSUPPORTED, "blocks must be in [1, 4096] (got %d)", blocks);
  if (reinterpret_cast<uintptr_t>(neighbors) % 16 != 0)
    return fail(BSA_ERR_INVALID_ARGUMENT, "neighbors must be 16-byte aligned");
  cudaError_t e = bsa::launch_frontier_mask(route, neighbors, planes, blocks, frontier, err_word,
                                            static_cast<cudaStream_t>(stream), sm_count());
  if (e != cudaSuccess) return cuda_fail(e, "bsa_frontier_mask launch");
  return ok();
}

int bsa_directional_update(const float* mass, const uint8_t* previous, const int32_t* neighbors,
                           const uint8_t* previous_frontier, int64_t planes, int32_t blocks,
                           float persistence, float min_ratio, float candidate_bonus,
                           float budget_scale, int32_t max_blocks, int32_t explore_count,
                           int32_t expand, int32_t sink_blocks, int32_t rows_per_group,
                           uint8_t* route_out, uint8_t* frontier_out, uint8_t* candidates,
                           uint8_t* exploration, uint8_t* dropped, uint8_t* added,
                           int32_t* counts, int32_t* indices, uint64_t* kept, int32_t* err_word,
                           void* stream) {
  if (mass == nullptr || previous == nullptr || neighbors == nullptr || route_out == nullptr ||
      candidates == nullptr)
    return fail(BSA_ERR_INVALID_ARGUMENT,
                "mass, previous, neighbors, route_out and candidates must not be null");
  if (planes < 0 || blocks <= 0 || blocks > 4096)
    return fail(BSA_ERR_UNSUPPORTED, "blocks must be in [1, 4096] (got %d)", blocks);
  if (reinterpret_cast<uintptr_t>(neighbors) % 16 != 0)
    return fail(BSA_ERR_INVALID_ARGUMENT, "neighbors must be 16-byte aligned");
  if (max_blocks < 1 || max_blocks > blocks)
    return fail(BSA_ERR_INVALID_ARGUMENT, "max_blocks must be in [1, blocks] (got %d)", max_blocks);
  if (explore_count < 0 || explore_count > blocks)
    return fail(BSA_ERR_INVALID_ARGUMENT, "explore_count must be in [0, blocks] (got %d)",
                explore_count);
  if (!(budget_scale > 0.f))
    return fail(BSA_ERR_INVALID_ARGUMENT, "budget_scale must be positive");
  if (kept != nullptr && (rows_per_group <= 0 || (planes * blocks) % rows_per_group != 0))
    return fail(BSA_ERR_INVALID_ARGUMENT, "rows must be a multiple of rows_per_group");
  bsa::DirectionalArgs a{};
  a.mass = mass;
  a.prev = previous;
  a.neighbors = neighbors;
  a.prev_frontier = previous_frontier;
  a.planes = planes;
  a.n = blocks;
  a.persistence = persistence;
  a.min_ratio = min_ratio;
  a.candidate_bonus = candidate_bonus;
  a.budget_scale = budget_scale;
  a.cap = max_blocks;
  a.explore_count = explore_count;
  a.expand = expand;
  a.sink_blocks = sink_blocks < 0 ? 0 : sink_blocks;
  a.rows_per_group = rows_per_group > 0 ? rows_per_group : 1;
  a.candidates = candidates;
  a.route_out = route_out;
  a.exploration = exploration;
  a.dropped = dropped;
  a.added = added;
  a.counts = counts;
  a.indices = indices;
  a.kept = reinterpret_cast<unsigned long long*>(kept);
  a.err_word = err_word;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t cells = static_cast<size_t>(planes) * blocks * blocks;
  cudaError_t e = cudaMemsetAsync(candidates, 0, cells, s);
  if (e == cudaSuccess && kept != nullptr)
    e = cudaMemsetAsync(kept, 0, sizeof(uint64_t) * (planes * blocks / a.rows_per_group), s);
  if (e != cudaSuccess) return cuda_fail(e, "bsa_directional_update memset");
  e = bsa::launch_directional_update(a, s, sm_count());
  if (e != cudaSuccess) return cuda_fail(e, "bsa_directional_update launch");
  if (frontier_out != nullptr) {
    e = bsa::launch_frontier_mask(route_out, neighbors, planes, blocks, frontier_out, err_word, s,
                                  sm_count());
    if (e != cudaSuccess) return cuda_fail(e, "bsa_directional_update frontier launch");
  }
  return ok();
}

int bsa_sampled_mass(const void* sampled_q, const void* sampled_k, int64_t batch, int64_t heads,
                     int32_t q_blocks, int32_t samples, int32_t head_dim,
                     const float* block_bias, float scale, int32_t round_bf16, float* mass,
                     int32_t* err_word, void* stream) {
  CUtensorMap tq, tk;
  bsa::MassArgs a;
  const int rc = sampled_mass_setup(sampled_q, sampled_k, batch, heads, q_blocks, samples,
                                    head_dim, block_bias, scale, round_bf16, mass, err_word, &tq,
                                    &tk, &a);
  if (rc != BSA_OK) return rc;
  cudaError_t e = bsa::launch_sampled_mass(tq, tk, a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "bsa_sampled_mass launch");
  return ok();
}

int64_t bsa_sampled_mass_workspace_bytes(int64_t batch, int64_t heads, int32_t q_blocks,
                                         int32_t samples) {
  if (batch <= 0 || heads <= 0 || q_blocks <= 0 || samples <= 0) return 0;
  if (bsa::sampled_mass_on_chip(q_blocks, samples)) return 0;   // kept on chip
  const int64_t n_rows = static_cast<int64_t>(q_blocks) * samples;
  return batch * heads * n_rows * (static_cast<int64_t>(q_blocks) + 1) * 4;
}

int bsa_sampled_mass_onepass(const void* sampled_q, const void* sampled_k, int64_t batch,
                             int64_t heads, int32_t q_blocks, int32_t samples, int32_t head_dim,
                             const float* block_bias, float scale, int32_t round_bf16,
                             float* workspace, int64_t workspace_bytes, float* mass,
                             int32_t* err_word, void* stream) {
  const int64_t need = bsa_sampled_mass_workspace_bytes(batch, heads, q_blocks, samples);
  if (need > 0 && (workspace == nullptr || workspace_bytes < need))
    return fail(BSA_ERR_INVALID_ARGUMENT, "workspace of %lld bytes needed (got %lld)",
                static_cast<long long>(need), static_cast<long long>(workspace_bytes));
  if (need > 0 && (reinterpret_cast<uintptr_t>(workspace) & 15))
    return fail(BSA_ERR_INVALID_ARGUMENT, "workspace must be 16-byte aligned");
  if (batch * heads > 65535) return fail(BSA_ERR_UNSUPPORTED, "batch * heads must be <= 65535");
  CUtensorMap tq, tk;
  bsa::MassArgs a;
  const int rc = sampled_mass_setup(sampled_q, sampled_k, batch, heads, q_blocks, samples,
                                    head_dim, block_bias, scale, round_bf16, mass, err_word, &tq,
                                    &tk, &a);
  if (rc != BSA_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (bsa::sampled_mass_on_chip(q_blocks, samples)) {
    cudaError_t e = bsa::launch_sampled_mass_on_chip(tq, tk, a, s);
    if (e != cudaSuccess) return cuda_fail(e, "bsa_sampled_mass_onepass launch");
    return ok();
  }
  if (samples <= 2) {
    // One or two keys per block: the two-pass kernel (the workspace is unused).
    cudaError_t e = bsa::launch_sampled_mass(tq, tk, a, s);
    if (e != cudaSuccess) return cuda_fail(e, "bsa_sampled_mass_onepass launch");
    return ok();
  }
  a.block_lse = workspace;
  a.row_lse = workspace + batch * heads * a.n_rows * q_blocks;
  cudaError_t e = bsa::launch_sampled_mass(tq, tk, a, s);
  if (e != cudaSuccess) return cuda_fail(e, "bsa_sampled_mass_onepass launch");
  e = bsa::launch_sampled_mass_reduce(a, s);
  if (e != cudaSuccess) return cuda_fail(e, "bsa_sampled_mass_onepass reduce launch");
  return ok();
}

int bsa_sampled_mass_noalloc(const void* q, const void* k, int64_t batch, int64_t tokens,
                             int64_t heads, int32_t head_dim, int32_t block, int32_t samples,
                             float scale, int32_t round_bf16, float* mass, int32_t* err_word,
                             void* stream) {
  if (q == nullptr || k == nullptr || mass == nullptr || err_word == nullptr)
    return fail(BSA_ERR_INVALID_ARGUMENT, "null pointer argument");
  if (head_dim != 128) return fail(BSA_ERR_UNSUPPORTED, "head_dim must be 128 (got %d)", head_dim);
  if (block != 32 && block != 64 && block != 128)
    return fail(BSA_ERR_UNSUPPORTED, "block must be 32, 64 or 128 (got %d)", block);
  if (samples != 1 && samples != 2 && samples != 4 && samples != 8 && samples != 16 &&
      samples != 32)
    return fail(BSA_ERR_UNSUPPORTED, "samples must be a power of two <= 32 (got %d)", samples);
  if (samples > block)
    return fail(BSA_ERR_INVALID_ARGUMENT, "samples (%d) exceed the block (%d)", samples, block);
  if (batch <= 0 || tokens <= 0 || heads <= 0 || batch > 65535 || heads > 65535)
    return fail(BSA_ERR_INVALID_ARGUMENT, "bad batch/tokens/heads");
  if ((reinterpret_cast<uintptr_t>(q) & 15) || (reinterpret_cast<uintptr_t>(k) & 15))
    return fail(BSA_ERR_INVALID_ARGUMENT, "q and k must be 16-byte aligned");
  const int64_t q_blocks = (tokens + block - 1) / block;
  if (q_blocks > 4096)
    return fail(BSA_ERR_UNSUPPORTED, "q_blocks must be in [1, 4096] (got %lld)",
                static_cast<long long>(q_blocks));
  const int64_t n_rows = q_blocks * samples;
  const int64_t bias_bytes = ((q_blocks * 4 + 255) / 256) * 256;
  const int64_t per_head = 2 * n_rows * head_dim * 2;
  const int64_t room = static_cast<int64_t>(bsa::kNoAllocScratchBytes) - bias_bytes;
  if (per_head > room)
    return fail(BSA_ERR_UNSUPPORTED,
                "%lld sampled rows need %lld scratch bytes per head; the static scratch holds "
                "%lld",
                static_cast<long long>(n_rows), static_cast<long long>(per_head + bias_bytes),
                static_cast<long long>(bsa::kNoAllocScratchBytes));
  const int64_t hc_max = room / per_head;
  // Scratch address, looked up once per device with that device current.
  static void* scratch_of[64] = {};
  static std::mutex scratch_mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "bsa_sampled_mass_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(BSA_ERR_UNSUPPORTED, "device ordinal %d >= 64", dev);
  // The kernels run on the caller's stream with the current device's scratch:
  // a stream of another device is refused rather than launched with the
  // wrong device's address.
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int stream_dev = dev;
  e = cudaStreamGetDevice(st, &stream_dev);
  if (e != cudaSuccess) return cuda_fail(e, "bsa_sampled_mass_noalloc: cudaStreamGetDevice");
  if (stream_dev != dev)
    return fail(BSA_ERR_INVALID_ARGUMENT,
                "the stream belongs to device %d but device %d is current", stream_dev, dev);
  // The address is cached for the life of the process; it does not survive
  // cudaDeviceReset of this device.
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(scratch_mu);
    if (scratch_of[dev] == nullptr) {
      e = bsa::noalloc_scratch(&scratch_of[dev]);
      if (e != cudaSuccess) {
        scratch_of[dev] = nullptr;
        return cuda_fail(e, "bsa_sampled_mass_noalloc: cudaGetSymbolAddress");
      }
    }
    scratch = scratch_of[dev];
  }
  // Key-block weights log(size / S) of flex.py:236-237 (full blocks, last block).
  const int64_t tail = tokens - (q_blocks - 1) * block;
  const float bias_full = logf(static_cast<float>(block) / static_cast<float>(samples));
  const float bias_tail = logf(static_cast<float>(tail) / static_cast<float>(samples));
  uint8_t* base = static_cast<uint8_t*>(scratch);
  for (int64_t b = 0; b < batch; ++b) {
    for (int64_t h0 = 0; h0 < heads; h0 += hc_max) {
      const int64_t hc = heads - h0 < hc_max ? heads - h0 : hc_max;
      const int64_t region = n_rows * hc * head_dim * 2;
      e = bsa::launch_gather_samples(q, k, tokens, heads, static_cast<int>(b),
                                     static_cast<int>(h0), static_cast<int>(hc), block, samples,
                                     static_cast<int>(q_blocks), bias_full, bias_tail, scratch, st);
      if (e != cudaSuccess) return cuda_fail(e, "bsa_sampled_mass_noalloc gather launch");
      CUtensorMap tq, tk;
      bool tm = false;
      int rc = encode_bhtd(&tq, base, 1, n_rows, hc, head_dim, n_rows * hc * head_dim,
                           hc * head_dim, head_dim, 128, &tm);
      if (rc != BSA_OK) return rc;
      rc = encode_bhtd(&tk, base + region, 1, n_rows, hc, head_dim, n_rows * hc * head_dim,
                       hc * head_dim, head_dim, 128, &tm);
      if (rc != BSA_OK) return rc;
      if (tm) return fail(BSA_ERR_UNSUPPORTED, "sampled rows must be row-major [rows, heads, D]");
      bsa::MassArgs a{};
      a.batch = 1;
      a.heads = hc;
      a.n_rows = n_rows;
      a.samples = samples;
      a.q_blocks = static_cast<int32_t>(q_blocks);
      a.scale = scale;
      a.round_bf16 = round_bf16;
      a.block_bias = reinterpret_cast<const float*>(base + 2 * region);
      a.mass_scale = 1.0f / static_cast<float>(samples);
      a.mass = mass + (b * heads + h0) * q_blocks * q_blocks;
      a.err_word = err_word;
      e = bsa::launch_sampled_mass(tq, tk, a, st);
      if (e != cudaSuccess) return cuda_fail(e, "bsa_sampled_mass_noalloc mass launch");
    }
  }
  return ok();
}

int bsa_exact_block_mass(const void* q, const void* k, int64_t batch, int64_t tokens,
                         int64_t heads, int32_t head_dim, int32_t block, float scale,
                         const float* lse, float* mass, int32_t* err_word, void* stream) {
  if (q == nullptr || k == nullptr || mass == nullptr || err_word == nullptr)
    return fail(BSA_ERR_INVALID_ARGUMENT, "null pointer argument");
  if (head_dim != 128) return fail(BSA_ERR_UNSUPPORTED, "head_dim must be 128 (got %d)", head_dim);
  if (block != 32 && block != 64 && block != 128)
    return fail(BSA_ERR_UNSUPPORTED, "block must be 32, 64 or 128 (got %d)", block);
  if (batch <= 0 || tokens <= 0 || heads <= 0 || batch > 65535 || heads > 65535)
    return fail(BSA_ERR_INVALID_ARGUMENT, "bad batch/tokens/heads");
  const int64_t blocks = (tokens + block - 1) / block;
  if (blocks > 4096) return fail(BSA_ERR_UNSUPPORTED, "at most 4096 blocks (got %lld)",
                                 static_cast<long long>(blocks));
  CUtensorMap tq, tk;
  bool tm = false;
  int rc = encode_bhtd(&tq, q, batch, tokens, heads, head_dim, tokens * heads * head_dim,
                       heads * head_dim, head_dim, 128, &tm);
  if (rc != BSA_OK) return rc;
  rc = encode_bhtd(&tk, k, batch, tokens, heads, head_dim, tokens * heads * head_dim,
                   heads * head_dim, head_dim, 128, &tm);
  if (rc != BSA_OK) return rc;
  bsa::MassArgs a{};
  a.batch = batch;
  a.heads = heads;
  a.n_rows = tokens;
  a.samples = block;
  a.q_blocks = static_cast<int32_t>(blocks);
  a.scale = scale;
  a.round_bf16 = 0;
  a.block_bias = nullptr;
  a.mass_scale = 1.0f;
  a.lse = lse;
  a.mass = mass;
  a.err_word = err_word;
  cudaError_t e = bsa::launch_sampled_mass(tq, tk, a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "bsa_exact_block_mass launch");
  return ok();
}

static int attention_launch(const char* name, const void* q, const void* k, const void* v,
                            int64_t batch, int64_t tokens, int64_t heads, int32_t head_dim,
                            int64_t in_stride_b, int64_t in_stride_t, int64_t in_stride_h,
                            const int32_t* counts, const int32_t* indices, int32_t route_cols,
                            int32_t route_has_batch, int32_t block, float scale, void* out,
                            int64_t out_stride_b, int64_t out_stride_t, int64_t out_stride_h,
                            float* lse, float* block_lse, int32_t* err_word, void* stream,
                            const int32_t* out_rows = nullptr,
                            const void* const* out_peers = nullptr, int32_t n_peers = 0,
                            int64_t peer_tokens = 0) {
  if (q == nullptr || k == nullptr || v == nullptr || out == nullptr || counts == nullptr ||
      indices == nullptr || err_word == nullptr)
    return fail(BSA_ERR_INVALID_ARGUMENT, "null pointer argument");
  if (head_dim != 128) return fail(BSA_ERR_UNSUPPORTED, "head_dim must be 128 (got %d)", head_dim);
  if (block != 64 && block != 128)
    return fail(BSA_ERR_UNSUPPORTED, "block must be 64 or 128 (got %d)", block);
  if (batch <= 0 || tokens <= 0 || heads <= 0 || batch > 65535 || heads > 65535)
    return fail(BSA_ERR_INVALID_ARGUMENT, "bad batch/tokens/heads");
  const int64_t qblocks = (tokens + block - 1) / block;
  if (qblocks > 0x7fffffff) return fail(BSA_ERR_UNSUPPORTED, "too many blocks");
  if (route_cols < qblocks)
    return fail(BSA_ERR_INVALID_ARGUMENT, "route_cols (%d) < key blocks (%lld)", route_cols,
                static_cast<long long>(qblocks));
  if ((reinterpret_cast<uintptr_t>(out) & 15) || ((out_stride_t * 2) & 15) ||
      ((out_stride_h * 2) & 15) || ((out_stride_b * 2) & 15))
    return fail(BSA_ERR_INVALID_ARGUMENT, "out must be 16-byte aligned with 16-byte strides");
  CUtensorMap tq, tk, tv;
  bool tmq = false, tmk = false, tmv = false;
  int rc = encode_bhtd(&tq, q, batch, tokens, heads, head_dim, in_stride_b, in_stride_t,
                       in_stride_h, block, &tmq);
  if (rc != BSA_OK) return rc;
  rc = encode_bhtd(&tk, k, batch, tokens, heads, head_dim, in_stride_b, in_stride_t, in_stride_h,
                   block, &tmk);
  if (rc != BSA_OK) return rc;
  rc = encode_bhtd(&tv, v, batch, tokens, heads, head_dim, in_stride_b, in_stride_t, in_stride_h,
                   block, &tmv);
  if (rc != BSA_OK) return rc;
  if (tmq) return fail(BSA_ERR_UNSUPPORTED, "token stride below head stride is not supported");
  bsa::AttnArgs a{};
  a.batch = batch;
  a.tokens = tokens;
  a.heads = heads;
  a.q_blocks = static_cast<int32_t>(qblocks);
  a.k_blocks = static_cast<int32_t>(qblocks);
  a.block = block;
  a.route_cols = route_cols;
  a.route_batch_stride = route_has_batch ? 1 : 0;
  a.counts = counts;
  a.indices = indices;
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.in_stride_b = in_stride_b;
  a.in_stride_t = in_stride_t;
  a.in_stride_h = in_stride_h;
  a.scale = scale;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.out_stride_b = out_stride_b;
  a.out_stride_t = out_stride_t;
  a.out_stride_h = out_stride_h;
  a.lse = lse;
  a.err_word = err_word;
  a.block_lse = block_lse;
  a.out_rows = out_rows;
  a.n_peer = n_peers;
  a.peer_tokens = peer_tokens;
  for (int d = 0; d < n_peers; ++d)
    a.out_peer[d] = static_cast<__nv_bfloat16*>(const_cast<void*>(out_peers[d]));
  cudaError_t e = bsa::launch_attention(tq, tk, tv, a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, name);
  return ok();
}

int bsa_attention_fwd(const void* q, const void* k, const void* v, int64_t batch, int64_t tokens,
                      int64_t heads, int32_t head_dim, int64_t in_stride_b, int64_t in_stride_t,
                      int64_t in_stride_h, const int32_t* counts, const int32_t* indices,
                      int32_t route_cols, int32_t route_has_batch, int32_t block, float scale,
                      void* out, int64_t out_stride_b, int64_t out_stride_t,
                      int64_t out_stride_h, float* lse, int32_t* err_word, void* stream) {
  return attention_launch("bsa_attention_fwd launch", q, k, v, batch, tokens, heads, head_dim,
                          in_stride_b, in_stride_t, in_stride_h, counts, indices, route_cols,
                          route_has_batch, block, scale, out, out_stride_b, out_stride_t,
                          out_stride_h, lse, nullptr, err_word, stream);
}

int bsa_attention_fwd_peers(const void* q, const void* k, const void* v, int64_t tokens,
                            int64_t heads, int32_t head_dim, int64_t in_stride_t,
                            int64_t in_stride_h, const int32_t* counts, const int32_t* indices,
                            int32_t route_cols, int32_t block, float scale,
                            const int32_t* out_rows, const void* const* out_peers,
                            int32_t n_peers, int64_t peer_tokens, int64_t out_stride_t,
                            int64_t out_stride_h, int32_t* err_word, void* stream) {
  if (out_peers == nullptr || n_peers < 1 || n_peers > bsa::kMaxPeers)
    return fail(BSA_ERR_INVALID_ARGUMENT, "1 to %d output peers needed (got %d)", bsa::kMaxPeers,
                n_peers);
  if (peer_tokens <= 0 || peer_tokens * n_peers != tokens)
    return fail(BSA_ERR_INVALID_ARGUMENT, "peers x peer_tokens must equal tokens");
  for (int d = 0; d < n_peers; ++d) {
    if (out_peers[d] == nullptr || (reinterpret_cast<uintptr_t>(out_peers[d]) & 15))
      return fail(BSA_ERR_INVALID_ARGUMENT, "output peer %d is null or not 16-byte aligned", d);
    if (out_peers[d] == q || out_peers[d] == k || out_peers[d] == v)
      return fail(BSA_ERR_INVALID_ARGUMENT, "output peers must not alias q, k or v");
  }
  return attention_launch("bsa_attention_fwd_peers launch", q, k, v, 1, tokens, heads, head_dim,
                          tokens * in_stride_t, in_stride_t, in_stride_h, counts, indices,
                          route_cols, 0, block, scale, const_cast<void*>(out_peers[0]), 0,
                          out_stride_t, out_stride_h, nullptr, nullptr, err_word, stream, out_rows,
                          out_peers, n_peers, peer_tokens);
}

int bsa_pull_rows(const void* const* peer_shards, int32_t n_peers, int64_t peer_tokens,
                  int64_t src_row_bytes, int64_t src_tensor_bytes, int64_t src_offset,
                  const int32_t* perm, int64_t tokens, int64_t row_bytes, void* const* dst,
                  int32_t* err_word, void* stream) {
  if (peer_shards == nullptr || dst == nullptr || err_word == nullptr)
    return fail(BSA_ERR_INVALID_ARGUMENT, "null pointer argument");
  if (n_peers < 1 || n_peers > bsa::kMaxPeers)
    return fail(BSA_ERR_INVALID_ARGUMENT, "1 to %d peers needed (got %d)", bsa::kMaxPeers,
                n_peers);
  if (peer_tokens <= 0 || peer_tokens * n_peers != tokens)
    return fail(BSA_ERR_INVALID_ARGUMENT, "peers x peer_tokens must equal tokens");
  if (row_bytes <= 0 || (row_bytes & 15) || (src_row_bytes & 15) || (src_tensor_bytes & 15) ||
      (src_offset & 15) || src_offset + row_bytes > src_row_bytes)
    return fail(BSA_ERR_INVALID_ARGUMENT, "row sizes and offsets must be 16-byte multiples "
                "and the pulled bytes must lie inside a token's row");
  if (src_offset < 0 || src_tensor_bytes < peer_tokens * src_row_bytes)
    return fail(BSA_ERR_INVALID_ARGUMENT, "a shard's Q, K and V (src_tensor_bytes apart) must "
                "not overlap: src_tensor_bytes >= peer_tokens x src_row_bytes");
  cudaError_t e = bsa::launch_pull_rows(peer_shards, n_peers, peer_tokens, src_row_bytes,
                                        src_tensor_bytes, src_offset, perm, tokens, row_bytes,
                                        dst, err_word, static_cast<cudaStream_t>(stream),
                                        sm_count());
  if (e != cudaSuccess) return cuda_fail(e, "bsa_pull_rows launch");
  return ok();
}

// CUDA IPC of device buffers between the processes of a head-parallel group.
typedef CUresult (*AddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

static AddressRangeFn address_range_fn() {
  static AddressRangeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<AddressRangeFn>(p);
  });
  return fn;
}

int bsa_ipc_export(const void* ptr, void* handle, int64_t* offset) {
  if (ptr == nullptr || handle == nullptr || offset == nullptr)
    return fail(BSA_ERR_INVALID_ARGUMENT, "null pointer argument");
  AddressRangeFn range = address_range_fn();
  if (range == nullptr) return fail(BSA_ERR_CUDA, "cuMemGetAddressRange is unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  const CUresult r = range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr));
  if (r != CUDA_SUCCESS) return fail(BSA_ERR_CUDA, "cuMemGetAddressRange failed (%d)", (int)r);
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return cuda_fail(e, "bsa_ipc_export");
  std::memcpy(handle, &h, sizeof(h));
  *offset = static_cast<int64_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return ok();
}

int bsa_ipc_import(const void* handle, int64_t offset, void** ptr) {
  if (handle == nullptr || ptr == nullptr || offset < 0)
    return fail(BSA_ERR_INVALID_ARGUMENT, "bad argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "bsa_ipc_import");
  *ptr = static_cast<char*>(base) + offset;
  return ok();
}

int bsa_ipc_release(void* ptr, int64_t offset) {
  if (ptr == nullptr || offset < 0) return fail(BSA_ERR_INVALID_ARGUMENT, "bad argument");
  const cudaError_t e = cudaIpcCloseMemHandle(static_cast<char*>(ptr) - offset);
  if (e != cudaSuccess) return cuda_fail(e, "bsa_ipc_release");
  return ok();
}

int bsa_attention_fwd_scatter(const void* q, const void* k, const void* v, int64_t batch,
                              int64_t tokens, int64_t heads, int32_t head_dim,
                              int64_t in_stride_b, int64_t in_stride_t, int64_t in_stride_h,
                              const int32_t* counts, const int32_t* indices, int32_t route_cols,
                              int32_t route_has_batch, int32_t block, float scale,
                              const int32_t* out_rows, void* out, int64_t out_stride_b,
                              int64_t out_stride_t, int64_t out_stride_h, float* lse,
                              int32_t* err_word, void* stream) {
  if (out_rows == nullptr) return fail(BSA_ERR_INVALID_ARGUMENT, "out_rows is null");
  if (out == q || out == k || out == v)
    return fail(BSA_ERR_INVALID_ARGUMENT, "out must not alias q, k or v (rows are permuted)");
  return attention_launch("bsa_attention_fwd_scatter launch", q, k, v, batch, tokens, heads,
                          head_dim, in_stride_b, in_stride_t, in_stride_h, counts, indices,
                          route_cols, route_has_batch, block, scale, out, out_stride_b,
                          out_stride_t, out_stride_h, lse, nullptr, err_word, stream, out_rows);
}

int bsa_attention_dense_block_mass(const void* q, const void* k, const void* v, int64_t batch,
                                   int64_t tokens, int64_t heads, int32_t head_dim,
                                   int64_t in_stride_b, int64_t in_stride_t, int64_t in_stride_h,
                                   float scale, void* out, int64_t out_stride_b,
                                   int64_t out_stride_t, int64_t out_stride_h, float* lse,
                                   float* block_lse, float* mass, int32_t* err_word,
                                   void* stream) {
  if (lse == nullptr || block_lse == nullptr || mass == nullptr)
    return fail(BSA_ERR_INVALID_ARGUMENT, "lse, block_lse and mass must not be null");
  const int64_t blocks = (tokens + 127) / 128;
  if (blocks > 4096) return fail(BSA_ERR_UNSUPPORTED, "at most 4096 blocks");
  // The dense instantiation reads no route; counts / indices only satisfy
  // the shared argument checks.
  static const int32_t kNoRoute[1] = {0};
  int rc = attention_launch("bsa_attention_dense_block_mass launch", q, k, v, batch, tokens,
                            heads, head_dim, in_stride_b, in_stride_t, in_stride_h, kNoRoute,
                            kNoRoute, static_cast<int32_t>(blocks), 0, 128, scale, out,
                            out_stride_b, out_stride_t, out_stride_h, lse, block_lse, err_word,
                            stream);
  if (rc != BSA_OK) return rc;
  cudaError_t e = bsa::launch_block_mass(block_lse, lse, batch, tokens, heads,
                                         static_cast<int32_t>(blocks), mass,
                                         static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "bsa_attention_dense_block_mass mass launch");
  return ok();
}

}  // extern "C"
