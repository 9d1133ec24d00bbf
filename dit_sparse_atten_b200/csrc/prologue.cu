// (f4) Attention prologue in one pass over HBM: RMSNorm of the Q and K
// projections over their H*D features, rotary embedding of Q and K, and the
// spatial reorder of Q, K and V into route-block order.
//
// Reference semantics (attention_backends/):
//   rms_norm    svg_ops.py:82-92 (CPU path): float32 x * rsqrt(mean(x^2) + eps)
//               * weight, stored as bf16; the mean follows the reference's CPU
//               summation order (route_common.cuh), rsqrt = IEEE 1 / sqrt.
//   apply_rope  svg_ops.py:193-204: channel pairs (2j, 2j + 1) of each head as
//               a complex number times the token's rotary factor (cos_j, sin_j),
//               in float64, stored as bf16 (through float32, as torch does).
//   caller      wan_diffusers.py:44-56 (norm, head split, RoPE), then the
//               backend's reorder spatial.py:86-93.
// Output row i of every tensor is input token perm[i].  One warp per output
// row; each tensor row is C = H * D contiguous bf16.
#include "route_common.cuh"

namespace bsa {
namespace {

constexpr int kPrologueThreads = 256;

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// float -> bf16 bits, round to nearest even (the conversion unit).
__device__ __forceinline__ uint32_t bf16_bits(float x) {
  return static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(x)));
}

// Normalise 8 features of one row in place: x * r (IEEE), * weight, to bf16.
__device__ __forceinline__ void norm8(float (&y)[8], float r, const float* __restrict__ weight,
                                      int c) {
  float wv[8] = {1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f};
  if (weight != nullptr) {
    const float4 w0 = __ldg(reinterpret_cast<const float4*>(weight) + 2 * c);
    const float4 w1 = __ldg(reinterpret_cast<const float4*>(weight) + 2 * c + 1);
    wv[0] = w0.x; wv[1] = w0.y; wv[2] = w0.z; wv[3] = w0.w;
    wv[4] = w1.x; wv[5] = w1.y; wv[6] = w1.z; wv[7] = w1.w;
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    float t = __fmul_rn(y[e], r);
    if (weight != nullptr) t = __fmul_rn(t, wv[e]);
    y[e] = __uint_as_float(bf16_bits(t) << 16);
  }
}

// Channel pair (re, im) times (c, s) in float64, through float32 to bf16
// bits (re in the low half).  re and im carry 8 significant bits and c, s
// 24, so re*c, im*s, re*s and im*c are exact in float64: one rounding of
// re*c - im*s (or re*s + im*c) by a fused multiply-add equals the
// reference's product-then-subtract (each product exact, one rounding).
__device__ __forceinline__ uint32_t rope_pair(float re_f, float im_f, double c, double s) {
  const double re = re_f, im = im_f;
  const float o_re = __double2float_rn(__fma_rn(re, c, -__dmul_rn(im, s)));
  const float o_im = __double2float_rn(__fma_rn(re, s, __dmul_rn(im, c)));
  return bf16_bits(o_re) | (bf16_bits(o_im) << 16);
}

__device__ __forceinline__ void unpack8(const uint4 in, float (&y)[8]) {
  const uint32_t w[4] = {in.x, in.y, in.z, in.w};
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    y[2 * p] = bf16_lo(w[p]);
    y[2 * p + 1] = bf16_hi(w[p]);
  }
}

__device__ __forceinline__ uint4 pack8(const float (&y)[8]) {
  uint32_t out[4];
#pragma unroll
  for (int p = 0; p < 4; ++p) out[p] = bf16_bits(y[2 * p]) | (bf16_bits(y[2 * p + 1]) << 16);
  return make_uint4(out[0], out[1], out[2], out[3]);
}

// The Q and K rows of one token (C = H * D features each) together: both
// sums of squares in one packed ordered-sum chain (each component in the
// reference's order), then one pass over 8-feature chunks that normalises
// Q and K and rotates both with the same rotary factors (loaded and
// widened to float64 once per pair).
__device__ void norm_rope_qk_rows(const __nv_bfloat16* __restrict__ q_src,
                                  const __nv_bfloat16* __restrict__ k_src,
                                  __nv_bfloat16* __restrict__ q_dst,
                                  __nv_bfloat16* __restrict__ k_dst, int C, int D,
                                  const PrologueArgs& a, const float* __restrict__ cos_t,
                                  const float* __restrict__ sin_t) {
  const int lane = threadIdx.x & 31;
  float rq = 1.f, rk = 1.f;
  if (a.norm_q || a.norm_k) {
    const unsigned short* qr = reinterpret_cast<const unsigned short*>(q_src);
    const unsigned short* kr = reinterpret_cast<const unsigned short*>(k_src);
    // 8 items of each row per lane loaded ahead of their in-order additions
    const float2 ss = torch_cpu_sum<8>(
        [qr, kr](int e) {
          const float2 x = make_float2(
              __uint_as_float(static_cast<uint32_t>(__ldg(qr + e)) << 16),
              __uint_as_float(static_cast<uint32_t>(__ldg(kr + e)) << 16));
          return __fmul2_rn(x, x);
        },
        C);
    const float n = static_cast<float>(C);
    if (a.norm_q) rq = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss.x, n), a.eps)));
    if (a.norm_k) rk = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss.y, n), a.eps)));
  }
  const uint4* q4 = reinterpret_cast<const uint4*>(q_src);
  const uint4* k4 = reinterpret_cast<const uint4*>(k_src);
  uint4* qd4 = reinterpret_cast<uint4*>(q_dst);
  uint4* kd4 = reinterpret_cast<uint4*>(k_dst);
  for (int c = lane; c < C / 8; c += 32) {
    float yq[8], yk[8];
    unpack8(__ldg(q4 + c), yq);
    unpack8(__ldg(k4 + c), yk);
    if (a.norm_q) norm8(yq, rq, a.weight_q, c);
    if (a.norm_k) norm8(yk, rk, a.weight_k, c);
    if (cos_t != nullptr) {
      const int j0 = ((c * 8) % D) >> 1;            // first channel pair of this chunk
      const float4 cs = __ldg(reinterpret_cast<const float4*>(cos_t + j0));
      const float4 sn = __ldg(reinterpret_cast<const float4*>(sin_t + j0));
      const float cv[4] = {cs.x, cs.y, cs.z, cs.w};
      const float sv[4] = {sn.x, sn.y, sn.z, sn.w};
      uint32_t oq[4], ok[4];
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const double c0 = cv[p], s0 = sv[p];
        oq[p] = rope_pair(yq[2 * p], yq[2 * p + 1], c0, s0);
        ok[p] = rope_pair(yk[2 * p], yk[2 * p + 1], c0, s0);
      }
      qd4[c] = make_uint4(oq[0], oq[1], oq[2], oq[3]);
      kd4[c] = make_uint4(ok[0], ok[1], ok[2], ok[3]);
    } else {
      qd4[c] = pack8(yq);
      kd4[c] = pack8(yk);
    }
  }
}

__global__ void __launch_bounds__(kPrologueThreads, 4) qkv_prologue_kernel(PrologueArgs a) {
  const int C = a.heads * a.head_dim;
  const int64_t rows = a.batch * a.tokens;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (kPrologueThreads / 32);
  for (int64_t row = blockIdx.x * static_cast<int64_t>(kPrologueThreads / 32) + (threadIdx.x >> 5);
       row < rows; row += warps) {
    const int64_t b = row / a.tokens;
    const int64_t i = row - b * a.tokens;
    int64_t t = a.perm != nullptr ? static_cast<int64_t>(__ldg(a.perm + i)) : i;
    if (t < 0 || t >= a.tokens) {             // bad permutation entry: report, skip
      if ((threadIdx.x & 31) == 0) atomicOr(a.err_word, kErrBadRoute);
      continue;
    }
    const int64_t in_off = b * a.in_stride_b + t * a.in_stride_t;
    const int64_t out_off = row * C;
    if ((threadIdx.x & 31) == 0) {
      // Whole Q and K rows into L2 at once: the ordered sums below then wait
      // on L2 rather than DRAM (rows are 16-byte aligned, C * 2 bytes long).
      const uint32_t bytes = static_cast<uint32_t>(C) * 2u;
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a.q_in + in_off), "r"(bytes)
                   : "memory");
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a.k_in + in_off), "r"(bytes)
                   : "memory");
    }
    const float* cos_t = a.rope_cos != nullptr ? a.rope_cos + t * (a.head_dim / 2) : nullptr;
    const float* sin_t = a.rope_sin != nullptr ? a.rope_sin + t * (a.head_dim / 2) : nullptr;
    norm_rope_qk_rows(a.q_in + in_off, a.k_in + in_off, a.q_out + out_off, a.k_out + out_off, C,
                      a.head_dim, a, cos_t, sin_t);
    const uint4* vs = reinterpret_cast<const uint4*>(a.v_in + in_off);
    uint4* vd = reinterpret_cast<uint4*>(a.v_out + out_off);
    for (int c = threadIdx.x & 31; c < C / 8; c += 32) __stcs(vd + c, __ldcs(vs + c));
  }
}

}  // namespace

cudaError_t launch_qkv_prologue(const PrologueArgs& a, cudaStream_t stream, int num_sms) {
  const int64_t rows = a.batch * a.tokens;
  if (rows == 0) return cudaSuccess;
  const int64_t want = (rows + kPrologueThreads / 32 - 1) / (kPrologueThreads / 32);
  const int64_t cap = static_cast<int64_t>(num_sms) * 8;
  qkv_prologue_kernel<<<static_cast<unsigned>(want < cap ? want : cap), kPrologueThreads, 0,
                        stream>>>(a);
  return cudaGetLastError();
}

}  // namespace bsa
