/*
 * bsa.h -- C ABI of the B200 routed block-sparse attention path (libbsa.so).
 *
 * Drop-in for the FlexAttention pieces of the reference study's `flex_reuse`
 * attention backend (yangshuo1230/DiT_Sparse_Atten, attention_backends/).
 * Every entry point:
 *   - takes plain device pointers, sizes and element strides (no framework
 *     types) and a CUDA stream (cudaStream_t passed as void*; NULL = legacy
 *     default stream);
 *   - is stream-ordered and asynchronous: it validates arguments, enqueues
 *     kernels and returns without synchronising;
 *   - allocates no memory: outputs and workspaces are caller-owned;
 *   - returns BSA_OK or a negative status; the message for the last failure on
 *     the calling thread is available from bsa_last_error().
 * Kernels that can detect bad data at run time (out-of-range route entries,
 * a bounded wait that timed out) OR a bit from BSA_DEVICE_* into the
 * caller-provided int32 `err_word` (device memory) instead of faulting.
 * Target: sm_100a (NVIDIA B200).
 */
#ifndef BSA_H_
#define BSA_H_

#include <stdint.h>

#if defined(__GNUC__)
#define BSA_API __attribute__((visibility("default")))
#else
#define BSA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define BSA_OK 0
#define BSA_ERR_INVALID_ARGUMENT (-1)
#define BSA_ERR_UNSUPPORTED (-2)
#define BSA_ERR_CUDA (-3)
#define BSA_ERR_NO_DEVICE (-4)

/* Bits a kernel ORs into err_word. */
#define BSA_DEVICE_WAIT_TIMEOUT 1 /* a bounded mbarrier wait gave up */
#define BSA_DEVICE_BAD_ROUTE 2    /* a CSR count / block id / permutation entry was out of range */
#define BSA_DEVICE_TMEM_ALLOC 4   /* tensor-memory allocation returned an unusable address */
#define BSA_DEVICE_SMEM_LAYOUT 8  /* the dynamic shared memory could not hold the kernel's layout */

/* Library version, major*10000 + minor*100 + patch. */
BSA_API int bsa_version(void);

/* Message describing the last failed call on this thread ("" if none). */
BSA_API const char* bsa_last_error(void);

/*
 * (c) Spatial reorder (gather of whole token rows).
 * For t < n_tensors (1..3), b < batch, i < tokens_out:
 *   dst[t][b, i, :] = src[t][b, perm[i], :]
 * where a token row is `row_bytes` contiguous bytes and rows are contiguous
 * per batch element ([batch, tokens, row_bytes]).  perm values must lie in
 * [0, tokens_in); out-of-range entries are skipped and flag BSA_DEVICE_BAD_ROUTE.
 * Pack is perm = layout permutation, unpack is perm = its inverse.
 * Replaces: attention_backends/layout_ops.py:86-125 (reorder_qkv) and
 *           attention_backends/spatial.py:82-93 (reorder / reorder_qkv / restore).
 */
BSA_API int bsa_reorder_rows(int32_t n_tensors, const void* const* src, void* const* dst,
                     const int32_t* perm, int64_t batch, int64_t tokens_out, int64_t tokens_in,
                     int64_t row_bytes, int32_t* err_word, void* stream);

/*
 * (e) Row gather with a destination map, for the head-parallel (Ulysses)
 * exchange: for t < n_tensors, b < batch, i < rows:
 *   dst[t][b, dst_rows[i], :] = src[t][b, src_rows[i], :]
 * with `row_bytes`-byte rows, [batch, tokens_in, row] sources and
 * [batch, tokens_dst, row] destinations.  Out-of-range entries of either map
 * are skipped and flag BSA_DEVICE_BAD_ROUTE.  It lays Q/K/V head chunks out
 * as the all-to-all's send buffer and scatters received output chunks back
 * into [tokens, heads, D] without strided copies.
 * Replaces: nothing in the reference, which runs on one device; the
 * exchange is this build's multi-GPU layer.
 */
BSA_API int bsa_gather_scatter_rows(int32_t n_tensors, const void* const* src, void* const* dst,
                                    const int32_t* src_rows, const int32_t* dst_rows,
                                    int64_t batch, int64_t rows, int64_t tokens_in,
                                    int64_t tokens_dst, int64_t row_bytes, int32_t* err_word,
                                    void* stream);

/*
 * CSR pack of a boolean route [rows, cols] (uint8 0/1): counts[r] = number of
 * selected columns; indices[r, :] = selected column ids ascending, then the
 * unselected ids ascending.  cols <= 4096.
 * Replaces: attention_backends/layout_ops.py:128-151 (pack_boolean_rows),
 *           attention_backends/flex.py:275-281 (_pack_route).
 */
BSA_API int bsa_pack_boolean_rows(const uint8_t* route, int64_t rows, int32_t cols, int32_t* counts,
                          int32_t* indices, void* stream);

/*
 * (b) Route selection from fp32 block mass [rows, cols] (cols <= 4096):
 *   1. if prev != NULL and persistence != 0:
 *        mass = mass + persistence * mean_row(mass) * prev          (flex.py:535-541)
 *   2. top-mass: sort the row descending (ties: lower block id first), keep the
 *      first min(#(cumsum < sum * target) + 1, max_blocks), where the caller
 *      computes max_blocks = max(1, ceil(cols * keep)) as the reference does
 *      (in double precision)                                       (flex.py:83-94)
 *   3. force columns [0, sink_blocks) on                           (flex.py:550-566)
 *   4. write route_out [rows, cols] uint8, counts [rows], indices [rows, cols]
 *      (CSR as bsa_pack_boolean_rows) and, per group of rows_per_group
 *      consecutive rows, kept[g] = number of selected blocks     (flex.py:473-493)
 * The float32 sums follow the reference's PyTorch CPU evaluation order, so the
 * route is bit-identical to the reference's from the same mass.  Any of
 * route_out / counts / indices / kept may be NULL.  kept is overwritten.
 */
BSA_API int bsa_route_select(const float* mass, const uint8_t* prev, int64_t rows, int32_t cols,
                     int32_t rows_per_group, float persistence, float target,
                     int32_t max_blocks, int32_t sink_blocks, uint8_t* route_out,
                     int32_t* counts, int32_t* indices, uint64_t* kept, void* stream);

/*
 * (f4) Attention prologue in one pass: for every output row i and batch b,
 * token t = perm[i] (t = i when perm is NULL) of the projections q_proj /
 * k_proj / v_proj (bf16 [batch, tokens, heads * head_dim], row strides in
 * elements) becomes row i of q_out / k_out / v_out (bf16 [batch, tokens,
 * heads, head_dim] contiguous):
 *   q, k: RMSNorm over heads * head_dim when norm_q / norm_k is set,
 *         x * rsqrt(mean(x^2) + eps) * weight in float32 (weight fp32, NULL
 *         for none), rounded to bf16; then, when rope_cos / rope_sin
 *         (fp32 [tokens, head_dim / 2]) are given, channel pairs (2j, 2j+1)
 *         of every head times (cos_j + i sin_j) of token t in float64,
 *         rounded to bf16;
 *   v:    copied.
 * Bit-identical to the reference's CPU path (its mean's summation order
 * included).  perm entries outside [0, tokens) set BSA_DEVICE_BAD_ROUTE and
 * their rows are not written.  head_dim % 8 == 0; all pointers 16-byte aligned.
 * Replaces: attention_backends/wan_diffusers.py:44-56 (norm_q / norm_k through
 *           svg_ops.rms_norm, svg_ops.py:82-92, and svg_ops.apply_rope,
 *           svg_ops.py:193-204) and the backend's reorder, spatial.py:86-93.
 */
BSA_API int bsa_qkv_prologue(const void* q_proj, const void* k_proj, const void* v_proj,
                             int64_t batch, int64_t tokens, int64_t heads, int32_t head_dim,
                             int64_t in_stride_b, int64_t in_stride_t, int32_t norm_q,
                             int32_t norm_k, const float* norm_q_weight,
                             const float* norm_k_weight, float eps, const float* rope_cos,
                             const float* rope_sin, const int32_t* perm, void* q_out,
                             void* k_out, void* v_out, int32_t* err_word, void* stream);

/*
 * (f3) Frontier of a route: frontier[p, q, k] = route[p, q, k] and some valid
 * neighbour t of q has route[p, t, k] == 0, or some valid neighbour t of k has
 * route[p, q, t] == 0.  route / frontier: uint8 0/1 [planes, blocks, blocks]
 * (a plane is one batch x head route); neighbors: int32 [blocks, 4], 16-byte
 * aligned, -1 = no neighbour (the spatial layout's block neighbours).  Ids
 * outside [-1, blocks) set BSA_DEVICE_BAD_ROUTE in err_word (may be NULL)
 * and count as "no neighbour".  blocks <= 4096.
 * Replaces: attention_backends/routing.py:10-43 (frontier_mask).
 */
BSA_API int bsa_frontier_mask(const uint8_t* route, const int32_t* neighbors, int64_t planes,
                              int32_t blocks, uint8_t* frontier, int32_t* err_word, void* stream);

/*
 * (f3) Directional frontier update of a route (the directional branch of the
 * sampled route update), per plane [blocks, blocks]:
 *   1. for every cell of previous_frontier (NULL: the frontier of previous),
 *      the unselected neighbour with the highest mass along Q and along K
 *      (first of equal maxima), eligible when finite and >= mass * min_ratio;
 *      candidates at (best q, k) [expand bit 1], (q, best k) [bit 2] and
 *      (best q, best k) when both are eligible [bit 4], minus previous;
 *   2. pool = previous | candidates; if explore_count > 0 the explore_count
 *      highest masses outside the pool join it (exploration);
 *   3. score = mass + persistence * mean(mass) * previous
 *                   [+ candidate_bonus * mean(mass) * candidates];
 *   4. keep the first clamp(ceil(#previous * budget_scale), 1, max_blocks),
 *      at most #pool and at least 1, pool cells of the score sorted
 *      descending (the reference's argsort tie order);
 *   5. dropped = previous & ~route, added = route & ~previous;
 *   6. force columns [0, sink_blocks) on; write route_out, the CSR (counts,
 *      indices as bsa_route_select) and kept per group of rows_per_group rows;
 *   7. frontier_out = frontier of route_out (as bsa_frontier_mask).
 * The caller computes max_blocks = max(1, ceil(blocks * keep)) and
 * explore_count = max(1, ceil(blocks * exploration_fraction)) (0 for none).
 * mass fp32 and all masks uint8 [planes, blocks, blocks]; candidates is
 * required (scratch and output); exploration / dropped / added / frontier_out /
 * counts / indices / kept may be NULL.  kept is overwritten.  Float sums follow
 * the reference's PyTorch CPU order: the route is bit-identical to the
 * reference's from the same inputs.
 * Replaces: attention_backends/routing.py:97-168 (directional_budget_update),
 *           attention_backends/flex.py:517-534 and :550-566 (caller and sink).
 */
BSA_API int bsa_directional_update(const float* mass, const uint8_t* previous,
                                   const int32_t* neighbors, const uint8_t* previous_frontier,
                                   int64_t planes, int32_t blocks, float persistence,
                                   float min_ratio, float candidate_bonus, float budget_scale,
                                   int32_t max_blocks, int32_t explore_count, int32_t expand,
                                   int32_t sink_blocks, int32_t rows_per_group,
                                   uint8_t* route_out, uint8_t* frontier_out, uint8_t* candidates,
                                   uint8_t* exploration, uint8_t* dropped, uint8_t* added,
                                   int32_t* counts, int32_t* indices, uint64_t* kept,
                                   int32_t* err_word, void* stream);

/*
 * (b) Sampled block mass.  sampled_q / sampled_k: bf16 [batch, q_blocks * samples,
 * heads, head_dim] contiguous (rows gathered with bsa_reorder_rows through the
 * sample token ids of flex.py:222-231).  block_bias: fp32 [q_blocks], the
 * per-key-block log(block_size_b / samples) of flex.py:236-237.  Writes
 * mass: fp32 [batch, heads, q_blocks, q_blocks].  samples in {1,2,4,8,16,32},
 * head_dim == 128, q_blocks <= 4096.  round_bf16 != 0 reproduces the bf16
 * score rounding of the reference (flex.py:245).
 * Replaces: attention_backends/flex.py:205-251 (_sampled_block_mass).
 */
BSA_API int bsa_sampled_mass(const void* sampled_q, const void* sampled_k, int64_t batch, int64_t heads,
                     int32_t q_blocks, int32_t samples, int32_t head_dim,
                     const float* block_bias, float scale, int32_t round_bf16, float* mass,
                     int32_t* err_word, void* stream);

/*
 * (b) Sampled block mass in one pass over the sampled keys: same inputs,
 * limits and output as bsa_sampled_mass (within float rounding).  Each
 * sampled query row keeps the log2 of its exponential sum over every key
 * block, with its running stabiliser folded in, as it streams the keys; once
 * its log-sum-exp is known, mass = mean over the block's query samples of
 * 2^(block - row).  With 16 or 32 samples and up to 473 blocks those values
 * stay on chip (TMEM and shared memory): bsa_sampled_mass_workspace_bytes
 * returns 0 and workspace may be NULL.  Other shapes write them to a caller
 * workspace of bsa_sampled_mass_workspace_bytes bytes (16-byte aligned) and
 * a second kernel forms the mass; samples <= 2 (one or two keys per block)
 * take the two-pass kernel, workspace unused.  The two-pass entry point
 * computes every score twice instead.
 * Replaces: attention_backends/flex.py:205-251 (_sampled_block_mass).
 */
BSA_API int64_t bsa_sampled_mass_workspace_bytes(int64_t batch, int64_t heads, int32_t q_blocks,
                                                 int32_t samples);
BSA_API int bsa_sampled_mass_onepass(const void* sampled_q, const void* sampled_k, int64_t batch,
                                     int64_t heads, int32_t q_blocks, int32_t samples,
                                     int32_t head_dim, const float* block_bias, float scale,
                                     int32_t round_bf16, float* workspace,
                                     int64_t workspace_bytes, float* mass, int32_t* err_word,
                                     void* stream);

/*
 * (b) Sampled block mass with no caller workspace; it allocates nothing.
 * No counterpart in the reference: it is bsa_sampled_mass for callers that
 * have no device allocator to take the sampled-row workspace from (a C or C++
 * host binding libbsa.so without PyTorch).  q, k: bf16 [batch, tokens, heads,
 * head_dim] contiguous; mass as bsa_sampled_mass.  The sample rows are gathered
 * from q and k (flex.py:222-231) into a 32 MiB static device scratch of the
 * library, a chunk of heads at a time; each head needs
 * 2 * q_blocks * samples * 256 bytes of it plus 4 * q_blocks, and larger
 * sizes are rejected with BSA_ERR_UNSUPPORTED.  Nothing has to be zeroed.
 * Calls on one device share the scratch: two calls must not be in flight at
 * the same time (on different streams or threads) or they race.  The first
 * call on a device looks up the scratch address (cudaGetSymbolAddress) and
 * configures the kernels, so make it before any stream capture; the address
 * is cached for the process and does not survive cudaDeviceReset.  The
 * stream must belong to the current device (else BSA_ERR_INVALID_ARGUMENT).
 * Same limits as bsa_sampled_mass (samples in {1,...,32}, head_dim == 128,
 * q_blocks <= 4096) and block in {32, 64, 128}.
 */
BSA_API int bsa_sampled_mass_noalloc(const void* q, const void* k, int64_t batch, int64_t tokens,
                                     int64_t heads, int32_t head_dim, int32_t block,
                                     int32_t samples, float scale, int32_t round_bf16, float* mass,
                                     int32_t* err_word, void* stream);

/*
 * (b) Exact dense block mass (the exact bootstrap / refresh route source):
 *   mass[b, h, qb, kb] = sum_{q in qb, k in kb, q,k < tokens} softmax_q(k)
 * over full-precision scores (no bf16 rounding) of q, k: bf16 [batch, tokens,
 * heads, head_dim] contiguous.  Writes fp32 [batch, heads, Qb, Qb].
 * block in {32, 64, 128}, head_dim == 128, Qb <= 4096.  lse: fp32 [batch,
 * heads, tokens], the natural-log log-sum-exp of each query row's scaled
 * scores (for example from bsa_attention_fwd over a full route), or NULL: then
 * the kernel computes it in a first pass over the keys.
 * Replaces: attention_backends/flex.py:97-108,167-202 (_block_attention_mass,
 *           given the LSE of the dense FlexAttention pass of flex.py:254-272).
 */
BSA_API int bsa_exact_block_mass(const void* q, const void* k, int64_t batch, int64_t tokens,
                         int64_t heads, int32_t head_dim, int32_t block, float scale,
                         const float* lse, float* mass, int32_t* err_word, void* stream);

/*
 * (a) Block-sparse attention forward.
 * q, k, v: bf16 [batch, tokens, heads, head_dim] with element strides
 * (in_stride_b, in_stride_t, in_stride_h) shared by q, k and v; the head_dim
 * stride is 1.  out: bf16 with its own strides.  Route: counts [RB, heads, Qb]
 * and indices [RB, heads, Qb, route_cols] int32 (CSR, first counts[] entries
 * used), Qb = ceil(tokens / block); RB = batch if route_has_batch else 1.
 * Query block qb of head h attends to all keys < tokens of the listed key
 * blocks; rows with an empty route produce zeros.  lse (optional, fp32
 * [batch, heads, tokens]) receives the natural-log row log-sum-exp.
 * block in {64, 128}; head_dim == 128; strides * 2 bytes multiple of 16.
 * Replaces: attention_backends/flex.py:358-399 (_flex_output/_flex_kernel over
 *           the BlockMask of flex.py:308-355).
 */
BSA_API int bsa_attention_fwd(const void* q, const void* k, const void* v, int64_t batch, int64_t tokens,
                      int64_t heads, int32_t head_dim, int64_t in_stride_b, int64_t in_stride_t,
                      int64_t in_stride_h, const int32_t* counts, const int32_t* indices,
                      int32_t route_cols, int32_t route_has_batch, int32_t block, float scale,
                      void* out, int64_t out_stride_b, int64_t out_stride_t,
                      int64_t out_stride_h, float* lse, int32_t* err_word, void* stream);

/*
 * (a) Block-sparse attention forward with the spatial unpack folded into the
 * output store: the same arguments as bsa_attention_fwd, plus out_rows
 * (int32 [tokens], a permutation): query row i (in the packed route-block
 * order of q, k and v) of every batch element is written to token out_rows[i]
 * of out.  With out_rows = the layout's pack permutation the output comes out
 * in the original (F, H, W) token order, so no separate unpack pass is needed.
 * out must not alias q, k or v.  lse, when given, stays in packed row order.
 * Ids outside [0, tokens) set BSA_DEVICE_BAD_ROUTE and their rows are not
 * written.
 * Replaces: attention_backends/flex.py:358-399 (_flex_output) followed by the
 *           output restore of flex.py:694-700 / spatial.py:86-93.
 */
BSA_API int bsa_attention_fwd_scatter(const void* q, const void* k, const void* v, int64_t batch,
                                      int64_t tokens, int64_t heads, int32_t head_dim,
                                      int64_t in_stride_b, int64_t in_stride_t,
                                      int64_t in_stride_h, const int32_t* counts,
                                      const int32_t* indices, int32_t route_cols,
                                      int32_t route_has_batch, int32_t block, float scale,
                                      const int32_t* out_rows, void* out, int64_t out_stride_b,
                                      int64_t out_stride_t, int64_t out_stride_h, float* lse,
                                      int32_t* err_word, void* stream);

/*
 * (a) + (e) Block-sparse attention of one CFG branch (batch 1) of a
 * head-parallel group, storing every output row straight into the output
 * shard of the rank that holds its token: packed row i is token
 * t = out_rows[i] (out_rows may be NULL: t = i), which belongs to rank
 * d = t / peer_tokens and is written to token t - d * peer_tokens of
 * out_peers[d] with strides (out_stride_t, out_stride_h) elements, head h of
 * this call at out_peers[d] + h * out_stride_h.  out_peers[d] is rank d's
 * buffer mapped into this process (bsa_ipc_import; this rank's own buffer
 * for d = its rank), n_peers * peer_tokens == tokens, n_peers <= 8.  The
 * stores cross NVLink while the kernel runs: the attention and the output
 * all-to-all of the Ulysses exchange are one kernel.  The caller joins the
 * ranks (a collective on the stream) before reading its shard.  q, k, v:
 * [tokens, heads, head_dim] with the given strides; route as
 * bsa_attention_fwd (one route for the batch).
 * Replaces: attention_backends/flex.py:358-399 (_flex_output) and the
 * restore of flex.py:694-700, on a head shard; the exchange has no
 * counterpart (the reference runs on one device).
 */
BSA_API int bsa_attention_fwd_peers(const void* q, const void* k, const void* v, int64_t tokens,
                                    int64_t heads, int32_t head_dim, int64_t in_stride_t,
                                    int64_t in_stride_h, const int32_t* counts,
                                    const int32_t* indices, int32_t route_cols, int32_t block,
                                    float scale, const int32_t* out_rows,
                                    const void* const* out_peers, int32_t n_peers,
                                    int64_t peer_tokens, int64_t out_stride_t,
                                    int64_t out_stride_h, int32_t* err_word, void* stream);

/*
 * (e) The input side of the head-parallel exchange as pulls over peer
 * memory: for every packed row i (token t = perm[i], or i when perm is NULL)
 * and each of Q, K, V (x = 0, 1, 2), row_bytes bytes are read from rank
 * p = t / peer_tokens's input shard peer_shards[p] at byte
 * x * src_tensor_bytes + (t - p * peer_tokens) * src_row_bytes + src_offset
 * and written to dst[x] + i * row_bytes.  A shard is [3, peer_tokens, H, D]
 * (Q, K, V of the rank's tokens, every head); src_offset selects this rank's
 * heads.  peer_shards[p] is rank p's shard mapped into this process
 * (bsa_ipc_import; this rank's own for p = its rank), n_peers <= 8, all
 * sizes and addresses 16-byte multiples, src_offset + row_bytes <=
 * src_row_bytes and src_tensor_bytes >= peer_tokens * src_row_bytes (else
 * BSA_ERR_INVALID_ARGUMENT, nothing launched).  The caller joins the ranks (a
 * collective) after writing its shard and before any rank pulls.  No
 * reference counterpart: it replaces an all-to-all plus the pack gather.
 */
BSA_API int bsa_pull_rows(const void* const* peer_shards, int32_t n_peers, int64_t peer_tokens,
                          int64_t src_row_bytes, int64_t src_tensor_bytes, int64_t src_offset,
                          const int32_t* perm, int64_t tokens, int64_t row_bytes,
                          void* const* dst, int32_t* err_word, void* stream);

/*
 * (e) CUDA IPC of a device buffer between the processes of a head-parallel
 * group.  bsa_ipc_export writes the 64-byte handle of the allocation holding
 * ptr and ptr's offset in it; bsa_ipc_import maps a handle exported by
 * another process into this process on the current device (peer access
 * enabled) and returns the pointer at offset; bsa_ipc_release unmaps it
 * (ptr and offset as returned / given).  No reference counterpart.
 */
BSA_API int bsa_ipc_export(const void* ptr, void* handle, int64_t* offset);
BSA_API int bsa_ipc_import(const void* handle, int64_t offset, void** ptr);
BSA_API int bsa_ipc_release(void* ptr, int64_t offset);

/*
 * (a) + (f1) Dense attention with its exact block mass, one attention pass:
 * out = softmax(q k^T * scale) v over all keys, lse = its natural-log
 * log-sum-exp per query row ([batch, heads, tokens]), and
 *   mass[b, h, qb, kb] = sum_{q in qb, k in kb} softmax_q(k)
 * ([batch, heads, Qb, Qb], 128-token blocks) as bsa_exact_block_mass with that
 * lse, without a second pass over the keys: the attention writes, per query
 * row and key block, the log2 of the block's exponential sum to block_lse
 * (fp32 workspace [batch, heads, Qb, tokens], contents on return unspecified)
 * and a reduction kernel normalises and sums them.  Inputs and out as
 * bsa_attention_fwd (head_dim 128); Qb <= 4096.
 * Replaces: attention_backends/flex.py:254-272 (_dense_bootstrap: dense
 *           FlexAttention with return_lse, then _block_attention_mass).
 */
BSA_API int bsa_attention_dense_block_mass(const void* q, const void* k, const void* v,
                                           int64_t batch, int64_t tokens, int64_t heads,
                                           int32_t head_dim, int64_t in_stride_b,
                                           int64_t in_stride_t, int64_t in_stride_h, float scale,
                                           void* out, int64_t out_stride_b, int64_t out_stride_t,
                                           int64_t out_stride_h, float* lse, float* block_lse,
                                           float* mass, int32_t* err_word, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* BSA_H_ */
