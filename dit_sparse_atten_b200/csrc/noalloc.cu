// Module-level scratch for the entry point that allocates nothing
// (bsa_sampled_mass_noalloc): the sampled Q/K rows of a chunk of heads and the
// per-key-block weights are gathered here, then the sampled-mass kernel reads
// them.  Every call writes all of the scratch it reads before reading it, so
// nothing has to start at zero; calls in flight at the same time on one device
// share the scratch and must not overlap.
#include "bsa_kernels.h"

namespace bsa {
namespace {

__device__ __align__(256) uint8_t g_sample_scratch[kNoAllocScratchBytes];

// One thread per 16-byte piece of a sampled row: tensor (q or k), row r of the
// N = Qb * S sampled rows, head hh of the chunk, piece v of 16 (D = 128 bf16).
// Sample s of block kb is token kb * block + min(floor((2s+1) * size / (2S)),
// size - 1), size = min(block, T - kb * block) (attention_backends/flex.py:
// 222-231).  Thread i < Qb also writes the block's weight log(size / S).
__global__ void gather_samples_kernel(const uint4* __restrict__ q, const uint4* __restrict__ k,
                                      int64_t T, int64_t H, int b, int h0, int hc, int block,
                                      int samples, int q_blocks, float bias_full, float bias_tail,
                                      uint4* __restrict__ dst_q, uint4* __restrict__ dst_k,
                                      float* __restrict__ bias) {
  const int64_t n_rows = static_cast<int64_t>(q_blocks) * samples;
  const int64_t per_tensor = n_rows * hc * 16;
  const int64_t total = 2 * per_tensor;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int tensor = i >= per_tensor;
    const int64_t e = tensor ? i - per_tensor : i;
    const int v = static_cast<int>(e & 15);
    const int64_t rh = e >> 4;              // r * hc + hh
    const int hh = static_cast<int>(rh % hc);
    const int64_t r = rh / hc;
    const int kb = static_cast<int>(r / samples);
    const int s = static_cast<int>(r % samples);
    const int64_t size = min(static_cast<int64_t>(block), T - static_cast<int64_t>(kb) * block);
    const int64_t local = min((2 * s + 1) * size / (2 * samples), size - 1);
    const int64_t token = static_cast<int64_t>(kb) * block + local;
    const int64_t src = ((b * T + token) * H + h0 + hh) * 16 + v;
    if (tensor == 0) {
      dst_q[e] = __ldg(q + src);
    } else {
      dst_k[e] = __ldg(k + src);
    }
    if (i < q_blocks) bias[i] = (i + 1 == q_blocks) ? bias_tail : bias_full;
  }
}

}  // namespace

cudaError_t noalloc_scratch(void** ptr) {
  return cudaGetSymbolAddress(ptr, g_sample_scratch);
}

cudaError_t launch_gather_samples(const void* q, const void* k, int64_t T, int64_t H, int b,
                                  int h0, int hc, int block, int samples, int q_blocks,
                                  float bias_full, float bias_tail, void* scratch,
                                  cudaStream_t stream) {
  const int64_t region = static_cast<int64_t>(q_blocks) * samples * hc * 256;  // bytes per tensor
  uint8_t* base = static_cast<uint8_t*>(scratch);
  const int64_t total = 2 * static_cast<int64_t>(q_blocks) * samples * hc * 16;
  const int threads = 256;
  const int64_t want = (total + threads - 1) / threads;
  const unsigned grid = static_cast<unsigned>(want < 4096 ? want : 4096);
  gather_samples_kernel<<<grid, threads, 0, stream>>>(
      static_cast<const uint4*>(q), static_cast<const uint4*>(k), T, H, b, h0, hc, block, samples,
      q_blocks, bias_full, bias_tail, reinterpret_cast<uint4*>(base),
      reinterpret_cast<uint4*>(base + region), reinterpret_cast<float*>(base + 2 * region));
  return cudaGetLastError();
}

}  // namespace bsa
