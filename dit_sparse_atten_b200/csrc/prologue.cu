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

// One tensor row: optional RMSNorm (weight may be null), optional RoPE, store.
__device__ void norm_rope_row(const __nv_bfloat16* __restrict__ src, __nv_bfloat16* __restrict__ dst,
                              int C, int D, bool norm, const float* __restrict__ weight, float eps,
                              const float* __restrict__ cos_t, const float* __restrict__ sin_t) {
  const int lane = threadIdx.x & 31;
  const unsigned short* raw = reinterpret_cast<const unsigned short*>(src);
  float r = 1.f;
  if (norm) {
    // 16 items per lane loaded ahead of their in-order additions
    const float ss = torch_cpu_sum<16>(
        [raw](int e) {
          const float x = __uint_as_float(static_cast<uint32_t>(__ldg(raw + e)) << 16);
          return __fmul_rn(x, x);
        },
        C);
    r = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(C)), eps)));
  }
  const uint4* s4 = reinterpret_cast<const uint4*>(src);
  uint4* d4 = reinterpret_cast<uint4*>(dst);
  for (int c = lane; c < C / 8; c += 32) {
    const uint4 in = __ldg(s4 + c);
    const uint32_t w[4] = {in.x, in.y, in.z, in.w};
    float y[8];
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      y[2 * p] = bf16_lo(w[p]);
      y[2 * p + 1] = bf16_hi(w[p]);
    }
    if (norm) {
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
    uint32_t out[4];
    if (cos_t != nullptr) {
      const int j0 = ((c * 8) % D) >> 1;            // first channel pair of this chunk
      const float4 cs = __ldg(reinterpret_cast<const float4*>(cos_t + j0));
      const float4 sn = __ldg(reinterpret_cast<const float4*>(sin_t + j0));
      const float cv[4] = {cs.x, cs.y, cs.z, cs.w};
      const float sv[4] = {sn.x, sn.y, sn.z, sn.w};
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const double re = y[2 * p], im = y[2 * p + 1];
        const double c0 = cv[p], s0 = sv[p];
        const float o_re = __double2float_rn(__dsub_rn(__dmul_rn(re, c0), __dmul_rn(im, s0)));
        const float o_im = __double2float_rn(__dadd_rn(__dmul_rn(re, s0), __dmul_rn(im, c0)));
        out[p] = bf16_bits(o_re) | (bf16_bits(o_im) << 16);
      }
    } else {
#pragma unroll
      for (int p = 0; p < 4; ++p) out[p] = bf16_bits(y[2 * p]) | (bf16_bits(y[2 * p + 1]) << 16);
    }
    d4[c] = make_uint4(out[0], out[1], out[2], out[3]);
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
    norm_rope_row(a.q_in + in_off, a.q_out + out_off, C, a.head_dim, a.norm_q, a.weight_q,
                  a.eps, cos_t, sin_t);
    norm_rope_row(a.k_in + in_off, a.k_out + out_off, C, a.head_dim, a.norm_k, a.weight_k,
                  a.eps, cos_t, sin_t);
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
